"""vLLM with this package's plugin against vLLM alone: the same engine and load, only the checks differ.

    python -m sdcguard_b200.tools.vllm_bench [--requests 256] [--new-tokens 128] [--steps 2] [--warmup 1]

Each arm is a child process (one vLLM engine each, in-process engine core so CUDA events see its work) serving the
headline load: the Qwen3-0.6B shape with random weights (vLLM's dummy loader, no tokenizer), prompts of 1024 to 2048
random token ids and 128 greedy tokens each, prefix caching off, 16-token KV blocks. The checked arm sets
SDCGUARD_B200=1 and registers `serve.vllm_plugin` before the engine is built, so every bf16 linear layer of the
model runs on the checked GEMM. Prints one JSON line: tokens/s of each arm (device time, CUDA events around the
timed generate() calls), the check overhead, the layers checked, the checks run and the alarms.

Reference: the reference's own stock path is vLLM with its plugin (src/sdcguard/vllm_plugin.py); this compares the
two check designs on one serving engine.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time

QWEN3_0_6B_HF = {
    "architectures": ["Qwen3ForCausalLM"], "model_type": "qwen3", "hidden_size": 1024, "intermediate_size": 3072,
    "num_hidden_layers": 28, "num_attention_heads": 16, "num_key_value_heads": 8, "head_dim": 128,
    "vocab_size": 151936, "max_position_embeddings": 40960, "rope_theta": 1000000.0, "rms_norm_eps": 1e-06,
    "tie_word_embeddings": True, "torch_dtype": "bfloat16", "hidden_act": "silu", "attention_bias": False,
    "attention_dropout": 0.0, "bos_token_id": 151643, "eos_token_id": 151645, "use_cache": True,
    "use_sliding_window": False, "max_window_layers": 28, "initializer_range": 0.02,
}


def child(a) -> None:
    import torch
    if a.child == "checked":
        os.environ["SDCGUARD_B200"] = "1"
        from ..serve import vllm_plugin
        vllm_plugin.register()
    from vllm import LLM, SamplingParams
    from vllm.inputs import TokensPrompt
    mdir = f"/tmp/sdcguard_b200_vllm_model_{os.getpid()}"
    os.makedirs(mdir, exist_ok=True)
    with open(os.path.join(mdir, "config.json"), "w") as f:
        json.dump(QWEN3_0_6B_HF, f)
    g = torch.Generator().manual_seed(1234)
    lens = torch.randint(a.min_prompt, a.max_prompt + 1, (a.requests,), generator=g).tolist()
    P = torch.randint(0, QWEN3_0_6B_HF["vocab_size"], (a.requests, max(lens)), generator=g)
    reqs = [TokensPrompt(prompt_token_ids=P[i, :lens[i]].tolist()) for i in range(a.requests)]
    sp = SamplingParams(max_tokens=a.new_tokens, min_tokens=a.new_tokens, ignore_eos=True, temperature=0.0)
    llm = LLM(model=mdir, load_format="dummy", skip_tokenizer_init=True, dtype="bfloat16", block_size=16,
              max_model_len=a.max_prompt + a.new_tokens, enable_prefix_caching=False, seed=0,
              gpu_memory_utilization=a.gpu_mem)
    first = None
    for _ in range(a.warmup):
        outs = llm.generate(reqs, sp, use_tqdm=False)
        first = first or [list(o.outputs[0].token_ids) for o in outs[:4]]
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record()
    for _ in range(a.steps):
        llm.generate(reqs, sp, use_tqdm=False)
    e1.record()
    torch.cuda.synchronize()
    wall = (time.perf_counter() - t0) / a.steps
    res = {"arm": a.child, "dev_ms": e0.elapsed_time(e1) / a.steps, "wall_ms": wall * 1e3,
           "tokens_per_step": sum(lens) + a.requests * a.new_tokens, "first_tokens": first}
    if a.child == "checked":
        from ..serve import vllm_plugin
        from . import _client
        res["coverage"] = vllm_plugin.coverage()
        m = _client.parse_metrics(vllm_plugin.metrics_text(torch.device("cuda", torch.cuda.current_device())))
        res["metrics"] = {k: m.get(k) for k in ("sdcguard_checks_total", "sdcguard_alarms_total",
                                                "sdcguard_layers_checked", "sdcguard_weights_checked_ratio",
                                                "sdcguard_polls_total", "sdcguard_generated_tokens_total")}
    print("VLLMRESULT " + json.dumps(res, default=str), flush=True)


def run_arm(arm: str, a) -> dict:
    env = dict(os.environ, VLLM_ENABLE_V1_MULTIPROCESSING="0", HF_HUB_OFFLINE="1", TRANSFORMERS_OFFLINE="1",
               VLLM_HOST_IP="127.0.0.1", SDCGUARD="0", SDCGUARD_B200="0")
    cmd = [sys.executable, "-m", "sdcguard_b200.tools.vllm_bench", "--child", arm, "--requests", str(a.requests),
           "--new-tokens", str(a.new_tokens), "--steps", str(a.steps), "--warmup", str(a.warmup),
           "--min-prompt", str(a.min_prompt), "--max-prompt", str(a.max_prompt), "--gpu-mem", str(a.gpu_mem)]
    p = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=a.timeout)
    if a.log_dir:
        os.makedirs(a.log_dir, exist_ok=True)
        with open(os.path.join(a.log_dir, f"vllm_{arm}.log"), "w") as f:
            f.write(p.stdout + "\n" + p.stderr)
    for line in p.stdout.splitlines():
        if line.startswith("VLLMRESULT "):
            return json.loads(line[len("VLLMRESULT "):])
    raise RuntimeError(f"{arm} arm failed (rc {p.returncode}): {p.stderr[-2000:]}")


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m sdcguard_b200.tools.vllm_bench")
    ap.add_argument("--child", choices=("checked", "unchecked"))
    ap.add_argument("--requests", type=int, default=256)
    ap.add_argument("--new-tokens", type=int, default=128)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--min-prompt", type=int, default=1024)
    ap.add_argument("--max-prompt", type=int, default=2048)
    ap.add_argument("--gpu-mem", type=float, default=0.85)
    ap.add_argument("--timeout", type=float, default=1200.0)
    ap.add_argument("--log-dir")
    a = ap.parse_args(argv)
    if a.child:
        child(a)
        return 0
    arms = {arm: run_arm(arm, a) for arm in ("unchecked", "checked")}
    tps = {k: v["tokens_per_step"] / (v["dev_ms"] / 1e3) for k, v in arms.items()}
    cov = arms["checked"].get("coverage") or {}
    devs = list((cov.get("devices") or {}).values())
    out = {"tool": "vllm_bench", "model": "Qwen3-0.6B shape, random weights", "requests": a.requests,
           "new_tokens": a.new_tokens, "checked_tokens_per_s": round(tps["checked"], 1),
           "unchecked_tokens_per_s": round(tps["unchecked"], 1),
           "overhead_pct": round(100.0 * (tps["unchecked"] / tps["checked"] - 1.0), 2),
           "layers_checked": cov.get("layers_checked"), "layers_left_out": cov.get("layers_left_out"),
           "checks": sum(d.get("checks", 0) for d in devs), "alarms": sum(d.get("alarms", 0) for d in devs),
           "unjudged": sum(d.get("unjudged", 0) for d in devs),
           "same_first_tokens": arms["checked"]["first_tokens"] == arms["unchecked"]["first_tokens"],
           "worker_metrics": arms["checked"].get("metrics")}
    print(json.dumps(out))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
