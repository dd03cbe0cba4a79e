"""Spot check kernel (sampled exact recompute of linear outputs) against its float64 restatement: a clean GEMM
output raises nothing, a flipped bit in a sampled output is reported at that (row, column), and the kernel's
decisions agree with the float64 scores."""
import pytest
import torch

from sdcguard_b200.numerics import abft
from sdcguard_b200.ops import gemm, spot

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _layer(m, n, k, bias, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    x = torch.randn(m, k, device=DEV, generator=g).bfloat16()
    w = (torch.randn(n, k, device=DEV, generator=g) * 0.02).bfloat16()
    b = (torch.randn(n, device=DEV, generator=g) * 0.1).bfloat16() if bias else None
    cw = gemm.CheckedWeight(w, b)
    table = gemm.StateTable(DEV, 4)
    y = gemm.checked_linear(x, cw, table.state, table.add("g (ABFT GEMM)", cw.nb))
    return x, w, None if b is None else b.float(), y, table


@pytest.mark.parametrize("bias", [False, True])
def test_clean_outputs_pass_and_agree_with_float64(bias):
    x, w, b, y, table = _layer(256, 4096, 1024, bias)
    slot = table.add("spot", 1, "rowblock")
    sched = spot.SpotSchedule(4096)
    for turn in range(4):
        rows, cols = sched.sample(256, turn, DEV)
        spot.spot_check(x, w, y, rows, cols, table.state[slot], bias=b)
    torch.cuda.synchronize()
    r = table.read(reset=True)[slot]
    assert r["z"] == 0.0 and r["checks"] == 4
    ref = spot.reference_scores(x, w, y, b)
    assert float(ref.max()) < 2.0        # the whole output is within the bound, not just the samples


def test_flipped_sampled_output_is_reported_where_it_is():
    x, w, b, y, table = _layer(64, 1024, 2048, False, seed=1)
    slot = table.add("spot", 1, "rowblock")
    rows = torch.arange(64, dtype=torch.int32, device=DEV)
    cols = torch.tensor([3, 200, 517, 999], dtype=torch.int32, device=DEV)
    yy = y.clone()
    # the lowest bf16 mantissa bit of a sampled output: far below its block's ABFT noise, one ulp of its own value
    yy.view(torch.int16)[17, 517] ^= 1
    spot.spot_check(x, w, yy, rows, cols, table.state[slot])
    torch.cuda.synchronize()
    r = table.read(reset=True)[slot]
    score = spot.reference_scores(x, w, yy)[17, 517].item()
    if score > 2.0:
        assert r["z"] > abft.Z_ALARM and r["flat"] == 17 * 1024 + 517
    else:
        assert r["z"] == 0.0
    # an exponent-bit flip is always seen
    yy = y.clone()
    yy.view(torch.int16)[5, 200] ^= 1 << 12
    spot.spot_check(x, w, yy, rows, cols, table.state[slot])
    torch.cuda.synchronize()
    r = table.read(reset=True)[slot]
    assert r["z"] > abft.Z_ALARM and r["flat"] == 5 * 1024 + 200
