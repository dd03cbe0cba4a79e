"""Operator and math-mode screens on the CPU: exact integer matmuls pass, a simulated wrong value fails with its
location, the math-mode noise model keeps clean results far below the alarm."""
import torch

from sdcguard_b200.tools import modes, screen_ops


def test_screen_ops_cpu_pass_and_simulated_failure():
    r = screen_ops.run(torch.device("cpu"), minutes=0, shapes=((64, 64, 0.25), (32, 128, 0.25)))
    assert r["verdict"] == "pass" and screen_ops.exit_code(r) == 0
    assert set(r["tests"]) == {"gemm_fp64", "gemm_fp32", "gemm_bf16"}
    assert "fma_fp32" in r["skipped"] and "memory" in r["skipped"]
    r = screen_ops.run(torch.device("cpu"), minutes=0, simulate="gemm_bf16", shapes=((64, 64, 0.25),))
    t = r["tests"]["gemm_bf16"]
    assert r["verdict"] == "FAIL" and screen_ops.exit_code(r) == 1 and t["wrong"] == 1
    assert t["first"][0]["element"] == 3 and t["first"][0]["shape"] == (64, 64, 512)


def test_math_modes_cpu_clean():
    r = modes.screen("cpu", shape=(128, 256, 256))
    assert r["verdict"] == "pass" and set(r["modes"]) == {"bf16", "fp32", "fp64"}
    assert all(m["worst_z"] < 1.0 for m in r["modes"].values()), r


def test_math_mode_judge_flags_one_wrong_value():
    g = torch.Generator().manual_seed(3)
    a = modes._exact("fp32", torch.randn(64, 128, generator=g))
    b = modes._exact("fp32", torch.randn(128, 256, generator=g))
    c = (a.float() @ b.float())
    assert modes.judge("fp32", a, b, c, False)["wrong_blocks"] == 0
    c[5, 200] *= 1.001
    r = modes.judge("fp32", a, b, c, False)
    assert r["wrong_blocks"] == 1 and r["z"] > modes.ALARM
