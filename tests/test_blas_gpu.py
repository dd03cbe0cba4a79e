"""cuBLASLt algorithm sweep and the burn-in cuBLAS calls through the native host probe, against float64."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
def test_sweep_every_algorithm_correct(dtype):
    from sdcguard_b200.tools.blas import sweep
    r = sweep(1024, 2048, 512, dtype)
    assert r["offered"] >= 1, r
    ok = [a for a in r["algorithms"] if a["status"] == 0]
    assert ok and all(a["unwritten"] == 0 for a in ok), r
    assert r["wrong_algorithms"] == [], r
    assert r["algorithms"][-1]["forced_1x1"]


def test_legacy_calls_and_fresh_memory():
    from sdcguard_b200.tools.blas import fresh_memory_nonzero, legacy
    r = legacy(512)
    assert all(v.get("verdict") == "pass" for v in r.values()), r
    assert fresh_memory_nonzero(1 << 20) >= 0
