"""Grouped block-scaled fp8 checked GEMM (all experts of a MoE layer in one launch): every expert's rows equal the
ungrouped fp8 GEMM of that expert bit for bit, rows past the tiles in use are not written, the check is clean, and
an injected accumulator flip is reported at its grouped row and block."""
import pytest
import torch

from sdcguard_b200.numerics import abft

pytestmark = pytest.mark.gpu


def test_grouped_fp8_matches_per_expert_and_checks():
    from sdcguard_b200.ops import fp8, gemm, moe
    dev = torch.device("cuda")
    E, H, N, T, K = 4, 512, 256, 100, 2
    g = torch.Generator(device=dev).manual_seed(21)
    x = torch.randn(T, H, device=dev, generator=g).bfloat16()
    ids = torch.stack([torch.randperm(E, device=dev, generator=g)[:K] for _ in range(T)]).int()
    ids[ids == 2] = 3                                     # expert 2 gets no rows
    ws = [(torch.randn(N, H, device=dev, generator=g) * 0.03).bfloat16() for _ in range(E)]
    grp = moe.Grouping(T, K, E, H, dev)
    xg, _ = grp.group(x, ids)
    stack = fp8.Fp8WeightStack(ws)
    xa = fp8.quantize_act(xg)
    table = gemm.StateTable(dev, 3)
    s0, s1, s2 = (table.add(n, stack.nb) for n in ("grouped (ABFT GEMM)", "per expert (ABFT GEMM)",
                                                    "inj (ABFT GEMM)"))
    out = torch.full((grp.cap, N), 7.0, dtype=torch.bfloat16, device=dev)
    fp8.checked_linear_fp8_grouped(xa, stack, grp.gband, grp.gcount, table.state, s0, out=out)
    torch.cuda.synchronize()
    rows = grp.expert_rows()
    assert rows[2][1] == 0
    for e, (a, n) in enumerate(rows):
        if n == 0:
            continue
        t0, t1 = a // 128, -(-(a + n) // 128)
        sub = fp8.Fp8Act(xa.q[a:a + n], xa.sa[a:a + n], xa.row_sq[a:a + n], xa.sf[t0:t1])
        ref = fp8.checked_linear_fp8(sub, stack.expert(e), table.state, s1)
        assert torch.equal(out[a:a + n], ref), e
    gc = int(grp.gcount.item())
    assert bool((out[gc * 128:] == 7.0).all())
    st = table.read(reset=True)
    assert st[s0]["z"] < 6 and st[s0]["unjudged"] == 0 and st[s0]["checks"] == 1
    a1 = rows[1][0]
    fp8.checked_linear_fp8_grouped(xa, stack, grp.gband, grp.gcount, table.state, s2, out=out,
                                   inject=(a1 + 1, 200, 1 << 29))
    torch.cuda.synchronize()
    flip = table.read(reset=True)[s2]
    assert flip["z"] > abft.Z_ALARM and flip["row"] == a1 + 1 and flip["block"] == 1
