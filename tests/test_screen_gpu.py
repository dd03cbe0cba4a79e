"""Operator screen on a B200: every test passes on a healthy GPU (library matmuls in seven precisions, this library's
own bf16 / fp8 tcgen05 kernels on exact inputs, realistic-data matmuls, CUDA-core FMAs, SM consistency, memory);
simulated wrong values in the native tests are reported with their location. Math modes clean."""
import pytest
import torch

from sdcguard_b200.tools import modes, screen_ops

pytestmark = pytest.mark.gpu

SMALL = dict(minutes=0, mem_share=0.02, mem_limit_gb=1.0, fma_n=1 << 20, sm_n=1 << 18,
             shapes=((256, 256, 0.5), (128, 512, 0.25)), real=((16, 1024, 1024),))


def test_screen_ops_all_pass():
    r = screen_ops.run(torch.device("cuda:0"), **SMALL)
    bad = {k: v for k, v in r["tests"].items() if v["verdict"] != "pass"}
    assert r["verdict"] == "pass" and not bad, (bad, r.get("error"))
    for name in ("gemm_sdc_bf16", "gemm_sdc_fp8", "fma_fp32", "fma_fp64", "sm_consistency", "memory"):
        assert name in r["tests"] and r["tests"][name]["checked"] > 0, (name, r["skipped"])
    assert r["tests"]["gemm_sdc_bf16"]["worst_score"] < 6


@pytest.mark.parametrize("test", ["fma_fp32", "fma_fp64", "sm_consistency", "memory"])
def test_screen_ops_simulated_native_failure(test):
    r = screen_ops.run(torch.device("cuda:0"), tests=[test], simulate=test, **SMALL)
    t = r["tests"][test]
    assert r["verdict"] == "FAIL" and t["wrong"] >= 1, r
    first = t["first"][0]
    assert first["element"] == {"fma_fp32": 5, "fma_fp64": 5, "sm_consistency": 9, "memory": 12345}[test]
    if test == "sm_consistency":
        assert len(first["sm"]) == 2


def test_math_modes_gpu_clean():
    r = modes.screen("cuda:0", shape=(512, 1024, 512))
    assert r["verdict"] == "pass", r
    assert len(r["modes"]) >= 5, r["skipped"]


def test_workload_screen_clean_then_simulated_failure_with_evidence(tmp_path):
    from sdcguard_b200.tools import screen
    r = screen.run("cuda:0", "tiny", minutes=0, rounds=1)
    assert r["verdict"] == "PASS" and r["checks"] > 0 and r["rounds"][0]["mismatched_tokens"] == 0, r
    r = screen.run("cuda:0", "tiny", minutes=0, rounds=1, simulate=True, out_dir=str(tmp_path))
    assert r["verdict"] == "FAIL" and r["failed_rounds"] == [0], r
    ev = r["rounds"][0]["evidence"]
    assert any("down" in str(e["detail"]) for e in r["rounds"][0]["events"]), r["rounds"][0]["events"]
    rp = screen.replay(ev)
    assert rp["reproducible"] is False and rp["alarms"] == 0, rp      # an injected flip does not come back


def test_check_card_is_valid_board_input():
    from sdcguard_b200.tools import board, check
    res = check.run("cuda:0", seconds=1.0, size=2048)
    c = check.card(res)
    c["minutes"] = 1.0          # the board counts cards of a minute or more; this test checks for one second
    c["digest"] = check.card_digest(c)
    assert board.validate(c) is None and c["result"] == "PASS", c
    assert len(c["fingerprint"]["output"]) == 32
