"""vLLM 0.22 serving the Qwen3-0.6B shape (random weights) on a B200 with this package's plugin: every bf16 linear
layer of the decoder runs on the checked GEMM inside vLLM's compiled, CUDA-graph-captured model, the checks run and
read clean, and greedy outputs match vLLM without the plugin on their first tokens (the GEMMs differ only in
rounding order)."""
import json
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu


def test_vllm_plugin_small_load(tmp_path):
    pytest.importorskip("vllm")
    p = subprocess.run([sys.executable, "-m", "sdcguard_b200.tools.vllm_bench", "--requests", "16", "--new-tokens",
                        "16", "--steps", "1", "--warmup", "1", "--min-prompt", "64", "--max-prompt", "256",
                        "--gpu-mem", "0.5", "--log-dir", str(tmp_path)], capture_output=True, text=True, timeout=1500)
    assert p.returncode == 0, p.stderr[-3000:]
    r = json.loads(p.stdout.strip().splitlines()[-1])
    assert r["layers_checked"] == 28 * 4, r
    assert r["checks"] > 0 and r["alarms"] == 0 and r["unjudged"] == 0, r
    assert r["checked_tokens_per_s"] > 0 and r["unchecked_tokens_per_s"] > 0
    wm = r["worker_metrics"]                  # what the worker's metrics exporter would publish
    assert wm["sdcguard_layers_checked"] == 112 and wm["sdcguard_checks_total"] > 0
    assert wm["sdcguard_generated_tokens_total"] > 0 and wm["sdcguard_alarms_total"] == 0
