"""The HTTP server on a B200 (tiny model, a subprocess) probed from outside: ready (with a probe request) says
PROTECTED, greedy outputs are isolated from their batch and decode agrees with prefill, streamed throughput and
latencies are measured; an unchecked server reads NOT PROTECTED; qualify serves a baseline and two candidates and
decides each: the same stack with the weight scan on is accepted with verified weights, the fp8 stack's arithmetic
and quantization checks ran clean."""
import json
import os
import socket
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _cmd(port, extra=""):
    return f"{sys.executable} -m sdcguard_b200.serve.http --model tiny --port {port} --max-num-seqs 16 " \
           f"--max-model-len 512 {extra}"


def test_server_probes(tmp_path):
    from sdcguard_b200.tools import consistency, isolation, perf, ready
    from sdcguard_b200.tools.qualify import Server
    os.chdir(ROOT)
    port = _port()
    url = f"http://127.0.0.1:{port}"
    srv = Server(_cmd(port), url, str(tmp_path / "s.log"))
    try:
        r = ready.check(url, probe=True)
        assert r["verdict"] == "PROTECTED", r
        assert isolation.run(url, probes=2, primers=3)["verdict"] == "NO LEAK SEEN"
        c = consistency.run(url, probes=2)
        assert c["verdict"] == "CONSISTENT", c
        p = perf.measure(url, perf.default_load(16), concurrency=4, max_tokens=8, rounds=2, warmup=2)
        assert p["complete"] and p["median"]["ttft_p50_ms"] > 0 and p["median"]["output_tokens_per_s"] > 0, p
    finally:
        srv.stop()
    port = _port()
    url = f"http://127.0.0.1:{port}"
    srv = Server(_cmd(port, "--unchecked"), url, str(tmp_path / "u.log"))
    try:
        assert ready.check(url, probe=True)["verdict"] == "NOT PROTECTED"
    finally:
        srv.stop()


def test_qualify_and_decide(tmp_path):
    from sdcguard_b200.tools import qualify
    os.chdir(ROOT)
    out = str(tmp_path / "q")
    args = "--model tiny --max-num-seqs 16 --max-model-len 512"
    pol = tmp_path / "policy.json"
    pol.write_text(json.dumps({"performance": {"required": False}}))
    rc = qualify.main(["--out", out, "--baseline", args, "--candidate", f"scan={args} --weight-scan-mb 4096",
                       "--candidate", f"fp8={args} --precision fp8", "--no-repeat-baseline", "--rounds", "2",
                       "--concurrency", "4", "--max-tokens", "8", "--quality-prompts", "4", "--policy", str(pol)])
    with open(os.path.join(out, "decision_scan.json")) as f:
        d = json.load(f)
    assert d["decision"] == "ACCEPT", d["why"]
    assert d["arithmetic"]["verdict"] == "NO FAULT OBSERVED" and d["weights"]["verdict"] == "VERIFIED", d["weights"]
    assert d["approximation"]["verdict"] == "WITHIN" and d["tested"]["longest_prompt"] > 0
    with open(os.path.join(out, "decision_fp8.json")) as f:
        f8 = json.load(f)
    assert f8["arithmetic"]["verdict"] == "NO FAULT OBSERVED", f8["arithmetic"]
    assert f8["quantization"]["verdict"] == "RIGHT", f8["quantization"]
    assert f8["scope"]["stacks"]["candidate"]["precision"] == "fp8"
    assert rc in (0, 1, 2) and os.path.exists(os.path.join(out, "report.txt"))
    assert os.path.exists(os.path.join(out, "repro_fp8.sh"))


def test_gate_model_same_stack_passes_and_fp8_is_scored():
    from sdcguard_b200.tools import gate_model
    ref = gate_model.reference("tiny", prompts=4, prompt_len=48, new=16)
    assert ref["recorded_is_top1"] > 0.9, ref["recorded_is_top1"]
    same = gate_model.check(ref)
    assert same["verdict"] == "PASS" and same["mean_kl"] < 1e-6 and same["top1_agreement"] == 1.0, same
    assert same["alarms"] == 0
    f8 = gate_model.check(ref, precision="fp8", noise=same)
    assert f8["mean_kl"] > 0 and f8["verdict"] in ("PASS", "WARN", "FAIL") and f8["alarms"] == 0, f8


def test_case_capture_replay_and_investigate(tmp_path):
    """A GEMM accumulator flip captured as a case: the recheck shows the output was wrong, replays on this GPU do
    not reproduce it, the casefile calls it a transient fault and investigate says NOT REPRODUCED."""
    import torch

    from sdcguard_b200.ops import gemm
    from sdcguard_b200.tools import casefile, investigate
    g = torch.Generator().manual_seed(0)
    x = torch.randn(256, 1024, generator=g).bfloat16().cuda()
    w = (torch.randn(512, 1024, generator=g) * 0.03).bfloat16().cuda()
    cw = gemm.CheckedWeight(w)
    st = gemm.StateTable("cuda:0", 2)
    slot = st.add("t", cw.nb)
    y = gemm.checked_linear(x, cw, st.state, slot, inject=(7, 300, 1 << 29))
    d = st.read()[0]
    assert d["row"] == 7 and d["block"] == 2
    case = casefile.capture(x, w, y, d["row"], d["block"])
    p = str(tmp_path / "case.pt")
    casefile.save(case, p)
    case = torch.load(p, weights_only=False)
    assert casefile.recheck(case)["output_wrong"]
    rep = casefile.replay(case, 12)
    assert not rep["reproduced"], rep
    cf = casefile.casefile(case, [rep])
    assert cf["outcome"] == "most consistent with: transient fault on the incident GPU", cf
    assert investigate.investigate(case, 4, ["cuda:0"])["verdict"] == "NOT REPRODUCED"
