"""The checked tcgen05 GEMM against a plain PyTorch fp32 reference of the same op: output values, clean
scores (no false alarm), detection and location of injected accumulator faults, and the state counters."""
import math

import pytest
import torch

from sdcguard_b200.numerics import abft

pytestmark = pytest.mark.gpu

SHAPES = [
    (128, 128, 64),
    (200, 384, 192),
    (256, 1024, 1024),
    (1000, 3072, 1024),
    (64, 4096, 1024),
    (1024, 1024, 3072),
    (333, 136, 520),
]


def _run(m, n, k, bn, bias=False, inject=None, seed=0):
    from sdcguard_b200.ops import gemm
    torch.manual_seed(seed)
    dev = torch.device("cuda")
    x = torch.randn(m, k, device=dev).to(torch.bfloat16)
    w = (torch.randn(n, k, device=dev) * 0.02).to(torch.bfloat16)
    b = torch.randn(n, device=dev) * 0.1 if bias else None
    cw = gemm.CheckedWeight(w, b)
    st = gemm.StateTable(dev, 4)
    slot = st.add("lin", cw.nb)
    y = gemm.checked_linear(x, cw, st.state, slot, bn=bn, inject=inject)
    torch.cuda.synchronize()
    return x, w, b, cw, st, y


@pytest.mark.parametrize("bn", [128, 256])
@pytest.mark.parametrize("m,n,k", SHAPES)
def test_output_matches_fp32_reference(m, n, k, bn):
    x, w, b, cw, st, y = _run(m, n, k, bn)
    ref = x.float() @ w.float().t()
    err = (y.float() - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert err <= 2 ** -7 * scale + 1e-3, (err, scale)
    d = st.read()[0]
    assert d["checks"] == 1
    assert d["unjudged"] == 0
    assert 0.0 < d["z"] < 2.0, d


@pytest.mark.parametrize("bn", [128, 256])
def test_bias_and_clean_score_matches_torch_model(bn):
    x, w, b, cw, st, y = _run(300, 640, 256, bn, bias=True)
    ref = x.float() @ w.float().t() + b
    assert (y.float() - ref).abs().max().item() < 2 ** -7 * ref.abs().max().item() + 1e-3
    d = st.read()[0]
    r = abft.reference_check(x, w, b, cw.cs)
    assert d["z"] < 2.0 and r["z"] < 2.0, (d, r["z"])


@pytest.mark.parametrize("bit", [30, 28, 25, 23, 22, 20, 31])
def test_injected_accumulator_flip_is_caught_and_located(bit):
    m, n, k = 512, 1024, 1024
    row = 301
    _, _, _, _, _, y0 = _run(m, n, k, 256)
    col = int(y0[row].float().abs().argmax())          # a large output: every listed bit moves it far
    x, w, b, cw, st, y = _run(m, n, k, 256, inject=(row, col, 1 << bit))
    d = st.read()[0]
    assert d["z"] > abft.Z_ALARM, d
    assert d["row"] == row and d["block"] == col // 128, d


def test_state_accumulates_over_calls():
    from sdcguard_b200.ops import gemm
    dev = torch.device("cuda")
    x = torch.randn(256, 512, device=dev).to(torch.bfloat16)
    w = (torch.randn(512, 512, device=dev) * 0.05).to(torch.bfloat16)
    cw = gemm.CheckedWeight(w)
    st = gemm.StateTable(dev, 2)
    s = st.add("a", cw.nb)
    for _ in range(5):
        gemm.checked_linear(x, cw, st.state, s)
    torch.cuda.synchronize()
    d = st.read()[0]
    assert d["checks"] == 5 and d["z"] < 2.0
    err = gemm.error_word(dev).item()
    assert err == 0


@pytest.mark.parametrize("bn", [128, 256])
@pytest.mark.parametrize("m,n,k", [(64, 1024, 4096), (256, 4096, 1024), (256, 1024, 3072)])
def test_split_k_small_m_output_check_seal_and_injection(bn, m, n, k):
    """Decode-sized M runs split over K where K is long (partial accumulators, then the reduce-and-judge
    kernel), and unsplit otherwise; both give the fused check's answers."""
    from sdcguard_b200.ops import gemm
    torch.manual_seed(3)
    dev = torch.device("cuda")
    x = torch.randn(m, k, device=dev).to(torch.bfloat16)
    w = (torch.randn(n, k, device=dev) * 0.02).to(torch.bfloat16)
    b = torch.randn(n, device=dev) * 0.1
    cw = gemm.CheckedWeight(w, b)
    st = gemm.StateTable(dev, 4)
    s0, s1 = st.add("clean", cw.nb), st.add("inj", cw.nb)
    seal = torch.empty(m, cw.nb, dtype=torch.int32, device=dev)
    y = gemm.checked_linear(x, cw, st.state, s0, bn=bn, seal=seal)
    ref = x.float() @ w.float().t() + b
    assert (y.float() - ref).abs().max().item() <= 2 ** -7 * ref.abs().max().item() + 1e-3
    assert torch.equal(seal, gemm.seal_reference(y))
    gemm.checked_linear(x, cw, st.state, s1, bn=bn, inject=(10, 700, 1 << 28))
    rows = st.read()
    assert rows[0]["checks"] == 1 and rows[0]["unjudged"] == 0 and rows[0]["z"] < 2.0, rows[0]
    assert rows[1]["z"] > abft.Z_ALARM and rows[1]["row"] == 10 and rows[1]["block"] == 5, rows[1]


@pytest.mark.parametrize("m,n,k", [(1, 128, 4096), (64, 640, 4096), (200, 1152, 3072), (7, 384, 16384)])
def test_split_k_odd_block_counts(m, n, k):
    """Split-K with an odd number of 128-column blocks: the partial accumulators' rows are padded to 16 bytes (the
    reduce kernel reads them as float4), so every shape the GEMM takes splits cleanly."""
    from sdcguard_b200.ops import gemm
    torch.manual_seed(5)
    dev = torch.device("cuda")
    x = torch.randn(m, k, device=dev).to(torch.bfloat16)
    w = (torch.randn(n, k, device=dev) * 0.02).to(torch.bfloat16)
    cw = gemm.CheckedWeight(w)
    st = gemm.StateTable(dev, 2)
    s0, s1 = st.add("clean", cw.nb), st.add("inj", cw.nb)
    y = gemm.checked_linear(x, cw, st.state, s0)
    ref = x.double() @ w.double().t()
    assert float((y.double() - ref).abs().max()) <= 2 ** -7 * float(ref.abs().max()) + 1e-3
    r, c = m - 1, n - 3
    gemm.checked_linear(x, cw, st.state, s1, inject=(r, c, 1 << 29))
    rows = st.read()
    assert rows[0]["z"] < 2.0 and rows[0]["unjudged"] == 0, rows[0]
    assert rows[1]["z"] > abft.Z_ALARM and rows[1]["row"] == r and rows[1]["block"] == c // 128, rows[1]
    assert gemm.error_word(dev).item() == 0


@pytest.mark.parametrize("m,n,k", [(768, 768, 16384), (384, 3072, 8192), (2304, 768, 16384), (3072, 768, 16384),
                                   (768, 3072, 16384), (1000, 768, 8192), (640, 256, 8192)])
def test_split_k_long_k_few_tiles(m, n, k):
    """Long-K GEMMs with few output tiles (training dW shapes) run as 256 x 256 CTA-pair tiles split over K (odd band
    counts and a ragged last band included): same output and check as unsplit."""
    from sdcguard_b200.ops import gemm
    torch.manual_seed(6)
    dev = torch.device("cuda")
    x = (torch.randn(m, k, device=dev) * 0.1).to(torch.bfloat16)
    w = torch.randn(n, k, device=dev).to(torch.bfloat16)
    cw = gemm.CheckedWeight(w)
    st = gemm.StateTable(dev, 2)
    s0, s1 = st.add("clean", cw.nb), st.add("inj", cw.nb)
    y = gemm.checked_linear(x, cw, st.state, s0)
    ref = x.double() @ w.double().t()
    assert float((y.double() - ref).abs().max()) <= 2 ** -7 * float(ref.abs().max()) + 1e-3
    assert gemm.pick_bn(m, n, k=k) == 256
    y128 = gemm.checked_linear(x, cw, st.state, s0, bn=128)          # 128-wide tiles, no pairs
    assert float((y128.double() - ref).abs().max()) <= 2 ** -7 * float(ref.abs().max()) + 1e-3
    gemm.checked_linear(x, cw, st.state, s1, inject=(m // 2, n // 3, 1 << 29))
    rows = st.read()
    assert rows[0]["z"] < 2.0 and rows[0]["unjudged"] == 0 and rows[0]["checks"] == 2, rows[0]
    assert rows[1]["z"] > abft.Z_ALARM and rows[1]["row"] == m // 2 and rows[1]["block"] == (n // 3) // 128
    assert gemm.error_word(dev).item() == 0


@pytest.mark.parametrize("m,k", [(5, 64), (300, 1000), (64, 4096), (768, 16384), (3, 20000), (2304, 16383)])
def test_row_sqnorm_matches_reference(m, k):
    """Row sums of squares (warp per row for short rows, a CTA per row for long ones, a ragged tail) against fp64."""
    from sdcguard_b200.ops import gemm
    dev = torch.device("cuda")
    kk = -(-k // 8) * 8
    base = torch.randn(m, kk, device=dev).to(torch.bfloat16)
    x = base[:, :k]                                   # row stride a multiple of 8, odd width allowed
    r = gemm.row_sqnorm(x)
    ref = x.double().pow(2).sum(1)
    assert float(((r.double() - ref).abs() / ref).max()) < 1e-4
