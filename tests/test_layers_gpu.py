"""Layer and attention kernels against plain PyTorch fp32 references of the same ops, and the exact replay
property the attention/norm checks rely on (a second run on sampled rows gives identical values)."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_add_rmsnorm_matches_fp32():
    from sdcguard_b200.ops import layers
    torch.manual_seed(0)
    for h in (1024, 4096, 2048):
        x = torch.randn(77, h, device=DEV).bfloat16()
        r = torch.randn(77, h, device=DEV).bfloat16()
        w = (1 + 0.1 * torch.randn(h, device=DEV)).bfloat16()
        res = r.clone()
        y, rs = layers.add_rmsnorm(x, w, 1e-6, residual=res, resid_out=res)
        hh = (x.float() + r.float()).bfloat16().float()
        ref = hh * torch.rsqrt(hh.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()
        assert torch.equal(res, hh.bfloat16())
        assert (y.float() - ref).abs().max().item() < 2 ** -7 * ref.abs().max().item()
        assert torch.allclose(rs, y.float().pow(2).sum(-1), rtol=1e-4)
        # replay of sampled rows from the stored residual stream is bit-exact
        rows = torch.tensor([0, 5, 76], dtype=torch.int32, device=DEV)
        y2, _ = layers.add_rmsnorm(res, w, 1e-6, rows=rows)
        assert torch.equal(y2, y[rows.long()])


def test_silu_mul_matches_fp32():
    from sdcguard_b200.ops import layers
    gu = torch.randn(33, 2 * 3072, device=DEV).bfloat16()
    out, rs = layers.silu_mul(gu)
    g, u = gu.float()[:, :3072], gu.float()[:, 3072:]
    ref = torch.nn.functional.silu(g) * u
    assert (out.float() - ref).abs().max().item() < 2 ** -7 * ref.abs().max().item() + 1e-3
    assert torch.allclose(rs, out.float().pow(2).sum(-1), rtol=1e-4)


def _rope_ref(x, pos, tab):
    c, s = tab[pos.long(), :, 0], tab[pos.long(), :, 1]          # (t, 64)
    x1, x2 = x[..., :64], x[..., 64:]
    return torch.cat([x1 * c[:, None] - x2 * s[:, None], x2 * c[:, None] + x1 * s[:, None]], -1)


def test_qk_norm_rope_kv_and_replay_check():
    from sdcguard_b200.ops import layers
    torch.manual_seed(1)
    nq, nkv, T = 16, 8, 40
    qkv = torch.randn(T, (nq + 2 * nkv) * 128, device=DEV).bfloat16()
    pos = torch.arange(100, 100 + T, device=DEV, dtype=torch.int32)
    nblocks = 8
    cache = torch.zeros(nblocks, 2, nkv, 16, 128, device=DEV, dtype=torch.bfloat16)
    slots = torch.arange(T, device=DEV, dtype=torch.int64) + 16     # blocks 1..3
    qn = (1 + 0.1 * torch.randn(128, device=DEV)).bfloat16()
    kn = (1 + 0.1 * torch.randn(128, device=DEV)).bfloat16()
    tab = layers.rope_table(4096, 128, 1e6, device=DEV)
    q = torch.empty(T, nq, 128, device=DEV, dtype=torch.bfloat16)
    layers.qk_norm_rope_kv(qkv, nq, nkv, pos, slots, qn, kn, 1e-6, tab, q, cache)
    x = qkv.float().view(T, nq + 2 * nkv, 128)

    def norm(v, w):
        n = (v * torch.rsqrt(v.pow(2).mean(-1, keepdim=True) + 1e-6)).bfloat16().float()
        return (n * w.float()).bfloat16().float()
    qr = _rope_ref(norm(x[:, :nq], qn), pos, tab)
    kr = _rope_ref(norm(x[:, nq:nq + nkv], kn), pos, tab)
    assert (q.float() - qr).abs().max().item() < 0.02 * qr.abs().max().item()
    kc = cache[1:4, 0].permute(0, 2, 1, 3).reshape(-1, nkv, 128)[:T]
    vc = cache[1:4, 1].permute(0, 2, 1, 3).reshape(-1, nkv, 128)[:T]
    assert (kc.float() - kr).abs().max().item() < 0.02 * kr.abs().max().item()
    assert torch.equal(vc, x[:, nq + nkv:].bfloat16())
    # replay in compare mode: clean -> no alarm; a flipped bit in the cache -> alarm
    st = torch.zeros(1, 4, dtype=torch.int64, device=DEV)
    rows = torch.tensor([0, 17, 39], dtype=torch.int32, device=DEV)
    layers.qk_norm_rope_kv(qkv, nq, nkv, pos, slots, qn, kn, 1e-6, tab, q, cache, rows=rows, check=st[0])
    torch.cuda.synchronize()
    assert st[0, 0].item() == 0 and st[0, 2].item() == 1
    cache.view(torch.int16)[2, 1, 3, 1, 5] ^= 1          # token 17 = block 2 offset 1, V head 3, dim 5
    layers.qk_norm_rope_kv(qkv, nq, nkv, pos, slots, qn, kn, 1e-6, tab, q, cache, rows=rows, check=st[0])
    torch.cuda.synchronize()
    assert (st[0, 0].item() >> 32) == 0x7F800000


def _paged_setup(lens, ctx_extra, nkv, seed=0):
    torch.manual_seed(seed)
    pages_per = [-(-(n + e) // 16) for n, e in zip(lens, ctx_extra)]
    total = sum(pages_per) + 4
    cache = torch.randn(total, 2, nkv, 16, 128, device=DEV).bfloat16() * 0.5
    perm = torch.randperm(total - 1, device=DEV)[: sum(pages_per)] + 1
    bt = torch.zeros(len(lens), max(pages_per), dtype=torch.int32, device=DEV)
    o = 0
    for r, n in enumerate(pages_per):
        bt[r, :n] = perm[o:o + n].int()
        o += n
    return cache, bt


def _gather_kv(cache, bt_row, n):
    pages = bt_row[: -(-n // 16)].long()
    k = cache[pages, 0].permute(0, 2, 1, 3).reshape(-1, cache.shape[2], 128)[:n]
    v = cache[pages, 1].permute(0, 2, 1, 3).reshape(-1, cache.shape[2], 128)[:n]
    return k, v


@pytest.mark.parametrize("nq,nkv", [(16, 8), (32, 8), (4, 1)])
def test_prefill_matches_reference_and_replays_exactly(nq, nkv):
    from sdcguard_b200.ops import attention, layers
    lens = [200, 77, 130]
    prior = [0, 40, 16]           # cached prefix tokens before the new ones
    cache, bt = _paged_setup(lens, prior, nkv)
    T = sum(lens)
    q = (torch.randn(T, nq, 128, device=DEV) * 0.5).bfloat16()
    pos, starts, s = [], [], 0
    for n, p0 in zip(lens, prior):
        starts.append(s)
        pos += list(range(p0, p0 + n))
        s += n
    pos_t = torch.tensor(pos, dtype=torch.int32, device=DEV)
    tiles = attention.prefill_tiles(starts, lens, nq // nkv).to(DEV)
    rs = torch.zeros(T, device=DEV)
    out = attention.prefill(q, cache, bt, pos_t, tiles, nq, nkv, row_sq=rs)
    torch.cuda.synchronize()
    for r, (n, p0) in enumerate(zip(lens, prior)):
        k, v = _gather_kv(cache, bt[r], p0 + n)
        ref = attention.reference_attention(q[starts[r]:starts[r] + n], k, v, pos_t[starts[r]:starts[r] + n].long())
        got = out[starts[r]:starts[r] + n].float()
        assert (got - ref).abs().max().item() < 0.02, (r, (got - ref).abs().max().item())
    assert torch.allclose(rs, out.float().pow(2).sum((1, 2)), rtol=1e-3)
    # replay of a sample of tokens on other CTAs: bit-exact
    sampled = [[starts[0] + 3, starts[0] + 150], [starts[1] + 76], [starts[2], starts[2] + 64, starts[2] + 129]]
    rt, ridx = attention.replay_tiles(sampled, nq // nkv)
    out2 = torch.zeros_like(out)
    attention.prefill(q, cache, bt, pos_t, rt.to(DEV), nq, nkv, out=out2, row_idx=ridx.to(DEV))
    torch.cuda.synchronize()
    for tok in ridx.tolist():
        assert torch.equal(out2[tok], out[tok]), tok
    st = torch.zeros(1, 4, dtype=torch.int64, device=DEV)
    flat = out.view(T, -1)
    layers.compare_rows(flat, ridx.to(DEV), out2.view(T, -1)[ridx.long()], st[0])
    torch.cuda.synchronize()
    assert st[0, 0].item() == 0
    out2.view(T, -1).view(torch.int16)[ridx[1].item(), 7] ^= 1
    layers.compare_rows(flat, ridx.to(DEV), out2.view(T, -1)[ridx.long()], st[0])
    torch.cuda.synchronize()
    assert (st[0, 0].item() >> 32) == 0x7F800000


@pytest.mark.parametrize("nq,nkv", [(16, 8), (32, 8), (4, 1), (64, 8), (8, 8)])
def test_decode_matches_reference_and_replays_exactly(nq, nkv):
    from sdcguard_b200.ops import attention
    ctxs = [1, 17, 300, 1029]
    cache, bt = _paged_setup(ctxs, [0] * 4, nkv, seed=3)
    B = len(ctxs)
    q = (torch.randn(B, nq, 128, device=DEV) * 0.5).bfloat16()
    ctx = torch.tensor(ctxs, dtype=torch.int32, device=DEV)
    req = torch.arange(B, dtype=torch.int32, device=DEV)
    out = attention.decode(q, cache, bt, req, ctx, nq, nkv, max_ctx=2048)
    torch.cuda.synchronize()
    for b, n in enumerate(ctxs):
        k, v = _gather_kv(cache, bt[b], n)
        ref = attention.reference_attention(q[b:b + 1], k, v, torch.tensor([n - 1], device=DEV))
        assert (out[b].float() - ref[0]).abs().max().item() < 0.02
    idx = torch.tensor([1, 3], dtype=torch.int32, device=DEV)
    out2 = torch.zeros_like(out)
    attention.decode(q, cache, bt, req, ctx, nq, nkv, max_ctx=2048, out=out2, seq_idx=idx)
    torch.cuda.synchronize()
    assert torch.equal(out2[idx.long()], out[idx.long()])


def _z_flat(st_row):
    from sdcguard_b200.numerics import abft
    d = abft.decode_state_row(st_row.cpu().tolist())
    return d["z"], d["flat"], d["checks"]


def test_in_kernel_replay_checks_clean_and_flipped():
    """Check mode of the norm, activation and attention kernels: recompute sampled rows and compare in place."""
    from sdcguard_b200.ops import attention, layers
    st = torch.zeros(8, 4, dtype=torch.int64, device=DEV)
    rows = torch.tensor([3, 17, 40], dtype=torch.int32, device=DEV)
    x = torch.randn(64, 1024, device=DEV).bfloat16()
    w = torch.ones(1024, device=DEV).bfloat16()
    y, _ = layers.add_rmsnorm(x, w, 1e-6)
    layers.add_rmsnorm(x, w, 1e-6, out=y, rows=rows, check=st[0])
    y.view(torch.int16)[17, 100] ^= 4
    layers.add_rmsnorm(x, w, 1e-6, out=y, rows=rows, check=st[1])
    gu = torch.randn(64, 2 * 512, device=DEV).bfloat16()
    a, _ = layers.silu_mul(gu)
    layers.silu_mul(gu, out=a, rows=rows, check=st[2])
    a.view(torch.int16)[40, 511] ^= 1
    layers.silu_mul(gu, out=a, rows=rows, check=st[3])
    # decode
    ctxs = [33, 300, 1029]
    nq, nkv = 16, 8
    cache, bt = _paged_setup(ctxs, [0] * 3, nkv, seed=4)
    q = (torch.randn(3, nq, 128, device=DEV) * 0.5).bfloat16()
    ctx = torch.tensor(ctxs, dtype=torch.int32, device=DEV)
    req = torch.arange(3, dtype=torch.int32, device=DEV)
    out = attention.decode(q, cache, bt, req, ctx, nq, nkv, max_ctx=2048)
    sel = torch.tensor([0, 2], dtype=torch.int32, device=DEV)
    attention.decode(q, cache, bt, req, ctx, nq, nkv, max_ctx=2048, out=out, seq_idx=sel, check=st[4])
    out.view(torch.int16)[2, 5, 7] ^= 1
    attention.decode(q, cache, bt, req, ctx, nq, nkv, max_ctx=2048, out=out, seq_idx=sel, check=st[5])
    # prefill
    lens = [100, 60]
    cache2, bt2 = _paged_setup(lens, [0, 0], nkv, seed=5)
    T = sum(lens)
    qp = (torch.randn(T, nq, 128, device=DEV) * 0.5).bfloat16()
    pos = torch.tensor(list(range(100)) + list(range(60)), dtype=torch.int32, device=DEV)
    tiles = attention.prefill_tiles([0, 100], lens, nq // nkv).to(DEV)
    op = attention.prefill(qp, cache2, bt2, pos, tiles, nq, nkv)
    rt, ridx = attention.replay_tiles([[5, 99], [130]], nq // nkv)
    attention.prefill(qp, cache2, bt2, pos, rt.to(DEV), nq, nkv, out=op, row_idx=ridx.to(DEV), check=st[6])
    op.view(torch.int16)[130, 3, 64] ^= 2
    attention.prefill(qp, cache2, bt2, pos, rt.to(DEV), nq, nkv, out=op, row_idx=ridx.to(DEV), check=st[7])
    torch.cuda.synchronize()
    for clean in (0, 2, 4, 6):
        z, _, n = _z_flat(st[clean])
        assert z == 0 and n == 1, (clean, z, n)
    assert _z_flat(st[1])[:2] == (math.inf, 17 * 1024 + 100)
    assert _z_flat(st[3])[:2] == (math.inf, 40 * 512 + 511)
    assert _z_flat(st[5])[:2] == (math.inf, 2 * nq * 128 + 5 * 128 + 7)
    assert _z_flat(st[7])[:2] == (math.inf, 130 * nq * 128 + 3 * 128 + 64)
