"""Grouped checked GEMM (all experts of a MoE layer in one launch, band -> expert table on the device): outputs
against a float64 product per expert, a clean check on clean data, an injected accumulator flip reported at its
grouped row and block, rows past the bands in use left alone, the layer against an fp32 PyTorch reference, and the
whole layer replayed from a CUDA graph."""
import pytest
import torch

pytestmark = pytest.mark.gpu

H, I, E, K = 512, 384, 6, 2


def _setup(T=200, seed=3):
    from sdcguard_b200.ops import gemm, moe
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(T, H, device=dev, generator=g).bfloat16()
    ids = torch.stack([torch.randperm(E, device=dev, generator=g)[:K] for _ in range(T)]).int()
    ids[:7] = torch.tensor([0, 1], dtype=torch.int32, device=dev)     # a busy expert pair
    ids[ids == 4] = 5                                                   # expert 4 gets no rows at all
    ws = [(torch.randn(2 * I, H, device=dev, generator=g) * 0.03).bfloat16() for _ in range(E)]
    grp = moe.Grouping(T, K, E, H, dev)
    return gemm, moe, dev, x, ids, ws, grp


def test_grouping_layout():
    gemm, moe, dev, x, ids, ws, grp = _setup()
    xg, rsq = grp.group(x, ids)
    torch.cuda.synchronize()
    rows = grp.expert_rows()
    gc = int(grp.gcount.item())
    assert rows[4][1] == 0
    assert sum(n for _, n in rows) == ids.numel()
    assert gc * 128 == sum(-(-n // 128) * 128 for _, n in rows)
    pos = grp.pos.view(-1, K).tolist()
    for t in range(x.shape[0]):
        for j in range(K):
            e = int(ids[t, j])
            r = pos[t][j]
            assert rows[e][0] <= r < rows[e][0] + rows[e][1]
            assert torch.equal(xg[r], x[t])
    for e, (a, n) in enumerate(rows):
        pad_end = a + -(-n // 128) * 128
        assert bool((xg[a + n:pad_end] == 0).all()) and bool((rsq[a + n:pad_end] == 0).all())
        for b in range(a // 128, pad_end // 128):
            assert int(grp.gband[b]) == e
    ref_sq = x.float().pow(2).sum(-1)
    r0 = pos[0][0]
    assert abs(float(rsq[r0]) - float(ref_sq[0])) < 1e-3 * float(ref_sq[0])


def test_grouped_gemm_matches_and_checks():
    gemm, moe, dev, x, ids, ws, grp = _setup()
    stack = gemm.CheckedWeightStack(ws)
    xg, rsq = grp.group(x, ids)
    table = gemm.StateTable(dev, 2)
    s0, s1 = table.add("clean (ABFT GEMM)", stack.nb), table.add("flip (ABFT GEMM)", stack.nb)
    out = torch.full((grp.cap, 2 * I), 7.0, dtype=torch.bfloat16, device=dev)
    gemm.checked_linear_grouped(xg, stack, grp.gband, grp.gcount, table.state, s0, row_sq=rsq, out=out)
    torch.cuda.synchronize()
    rows = grp.expert_rows()
    gc = int(grp.gcount.item())
    for e, (a, n) in enumerate(rows):
        if n == 0:
            continue
        ref = xg[a:a + n].double() @ ws[e].double().t()
        rel = ((out[a:a + n].double() - ref).abs() / (ref.abs() + 1e-2)).max().item()
        assert rel < 2 ** -7, (e, rel)
    assert bool((out[gc * 128:] == 7.0).all())          # rows past the bands in use are not written
    clean = table.read(reset=True)[s0]
    assert clean["z"] < 6 and clean["unjudged"] == 0 and clean["checks"] == 1
    # a flipped exponent bit in an accumulator of expert 1's second row
    a1 = rows[1][0]
    gemm.checked_linear_grouped(xg, stack, grp.gband, grp.gcount, table.state, s1, row_sq=rsq, out=out,
                                inject=(a1 + 1, 300, 1 << 29))
    torch.cuda.synchronize()
    flip = table.read(reset=True)[s1]
    assert flip["z"] > 6 and flip["row"] == a1 + 1 and flip["block"] == 300 // 128


def test_moe_layer_local_and_graph():
    from sdcguard_b200.models.moe import MoELayer, reference_moe
    dev = torch.device("cuda")
    T, Hm, Im, Em, Km = 96, 512, 256, 8, 2
    layer = MoELayer(Hm, Im, Em, Km, None, dev, checked=True, seed=5, collective="local")
    g = torch.Generator(device=dev).manual_seed(9)
    x = torch.randn(T, Hm, device=dev, generator=g).bfloat16()
    y = layer.forward(x)
    torch.cuda.synchronize()
    ref, _ = reference_moe(x, 5, Hm, Im, Em, Km, layer.last_ids, layer.last_wts)
    err = ((y.float() - ref).abs().max() / ref.abs().max()).item()
    assert err < 0.02, err
    rows = layer.state.read(reset=True)
    assert all(r["z"] < 6 and r["unjudged"] == 0 for r in rows)
    assert sum(r["checks"] for r in rows if "experts" in r["name"]) == 2
    # one CUDA graph holds the whole layer: no host read-back anywhere in it
    xs = x.clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        layer.forward(xs)                     # warm-up on the capture stream (buffers exist before capture)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        yg = layer.forward(xs)
    x2 = torch.randn(T, Hm, device=dev, generator=g).bfloat16()
    xs.copy_(x2)
    graph.replay()
    torch.cuda.synchronize()
    y2 = layer.forward(x2)
    torch.cuda.synchronize()
    assert torch.equal(yg, y2)
    layer.state.read(reset=True)
    del graph


def test_moe_layer_fp8_experts():
    """Block-scaled fp8 expert GEMMs: the layer against the fp32 reference within fp8's rounding, clean checks and
    quantization replays, and an injected accumulator flip in the gate/up GEMM found at its grouped row."""
    from sdcguard_b200.models.moe import MoELayer, reference_moe
    dev = torch.device("cuda")
    T, Hm, Im, Em, Km = 96, 512, 256, 8, 2
    layer = MoELayer(Hm, Im, Em, Km, None, dev, checked=True, seed=5, collective="local", precision="fp8")
    g = torch.Generator(device=dev).manual_seed(9)
    x = torch.randn(T, Hm, device=dev, generator=g).bfloat16()
    y = layer.forward(x)
    torch.cuda.synchronize()
    ref, _ = reference_moe(x, 5, Hm, Im, Em, Km, layer.last_ids, layer.last_wts)
    err = float((y.float() - ref).norm() / ref.norm())
    assert err < 0.08, err
    rows = {r["name"]: r for r in layer.state.read(reset=True)}
    assert all(r["z"] < 6 and r["unjudged"] == 0 for r in rows.values()), rows
    assert sum(r["checks"] for n, r in rows.items() if "fp8 GEMM" in n) == 2
    assert sum(r["checks"] for n, r in rows.items() if ".quant" in n) > 0
    layer.inject_next("up", 5, 200, 29)
    layer.forward(x)
    torch.cuda.synchronize()
    rows = {r["name"]: r for r in layer.state.read(reset=True)}
    up = [r for n, r in rows.items() if "gate_up (ABFT fp8" in n][0]
    assert up["z"] > 6 and up["row"] == 5 and up["block"] == 200 // 128, up
