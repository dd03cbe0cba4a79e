"""Tensor-parallel decoder: TP=1 prefill logits against a plain PyTorch fp32 forward of the same weights; TP=2
(two processes, skipped with fewer than 2 GPUs) against TP=1 (the chunked weight init gives the same global model
at any TP size); the checks stay clean and an injected flip in a reduce-scatter transfer is reported."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _meta(lens, tokens, dev, pages_per_seq, group):
    from sdcguard_b200.models.decoder import StepMeta
    from sdcguard_b200.ops import attention
    pos, slots, starts, last = [], [], [], []
    t0 = 0
    bt = torch.zeros(len(lens), pages_per_seq, dtype=torch.int32)
    for r, n in enumerate(lens):
        pages = list(range(1 + r * pages_per_seq, 1 + (r + 1) * pages_per_seq))
        bt[r] = torch.tensor(pages, dtype=torch.int32)
        starts.append(t0)
        pos.extend(range(n))
        slots.extend(pages[p // 16] * 16 + p % 16 for p in range(n))
        t0 += n
        last.append(t0 - 1)
    return StepMeta(mode="prefill", tokens=tokens.to(dev), pos=torch.tensor(pos, dtype=torch.int32, device=dev),
                    slots=torch.tensor(slots, dtype=torch.int64, device=dev), block_table=bt.to(dev),
                    logits_rows=torch.tensor(last, dtype=torch.int64, device=dev),
                    tiles=attention.prefill_tiles(starts, lens, group).to(dev))


def _prefill_logits(world, rank, lens, tokens, inject=False):
    from sdcguard_b200.models.decoder import TINY
    from sdcguard_b200.models.tp_decoder import TPDecoder
    from sdcguard_b200.parallel.symm import LocalHeap, SymmetricHeap
    from sdcguard_b200.parallel.tp import TPComm
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    heap = SymmetricHeap(device=dev) if world > 1 else LocalHeap(dev)
    comm = TPComm(heap, 512, TINY.hidden)
    m = TPDecoder(TINY, comm, rank, world, dev, checked=True, collective="own", max_rows=512, seed=3)
    m.buffers(512)
    pps = -(-max(lens) // 16)
    cache = torch.zeros(TINY.layers, 1 + len(lens) * pps, 2, m.nkv, 16, 128, dtype=torch.bfloat16, device=dev)
    meta = _meta(lens, tokens, dev, pps, m.nq // m.nkv)
    logits = m.forward(meta, cache)
    full = logits
    if world > 1:
        import torch.distributed as dist
        parts = [torch.empty_like(logits) for _ in range(world)]
        dist.all_gather(parts, logits.contiguous())
        full = torch.cat(parts, dim=1)
    torch.cuda.synchronize(dev)
    rows = m.read_checks(reset=True)
    alarms = [r for r in rows if r["z"] > 6]
    checks = sum(r["checks"] for r in rows)
    hit = None
    if inject:
        if rank == world - 1:
            comm.inject_next(0, 5, 3)
        m.forward(meta, cache)
        torch.cuda.synchronize(dev)
        hit = [(r["name"], r.get("row"), r.get("block"), r.get("peer")) for r in m.read_checks(reset=True)
               if r["z"] > 6]
    comm.close()
    return full.float().cpu(), alarms, checks, hit, m


def _reference(m, lens, tokens):
    """fp32 forward of the TP=1 model's weights (causal attention per sequence, GQA, q/k norm, rotate-half RoPE)."""
    cfg = m.cfg
    eps, d = cfg.rms_eps, cfg.head_dim

    def rms(x, w):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w.float()

    tab = m.rope.cpu()
    outs = []
    t0 = 0
    for n in lens:
        ids = tokens[t0:t0 + n]
        t0 += n
        pos = torch.arange(n)
        c, s = tab[pos, :, 0], tab[pos, :, 1]

        def rope(x):
            x1, x2 = x[..., :64], x[..., 64:]
            return torch.cat([x1 * c[:, None] - x2 * s[:, None], x2 * c[:, None] + x1 * s[:, None]], -1)

        h = m.embed.float().cpu()[ids]
        for lw in m.layers:
            y = rms(h, lw.ln1.cpu())
            qkv = y @ lw.qkv.float().cpu().t()
            nq, nkv = m.nq, m.nkv
            q = qkv[:, :nq * d].view(n, nq, d)
            k = qkv[:, nq * d:(nq + nkv) * d].view(n, nkv, d)
            v = qkv[:, (nq + nkv) * d:].view(n, nkv, d)
            if lw.q_norm is not None:
                q, k = rms(q, lw.q_norm.cpu()), rms(k, lw.k_norm.cpu())
            q, k = rope(q), rope(k)
            g = nq // nkv
            k, v = k.repeat_interleave(g, 1), v.repeat_interleave(g, 1)
            sc = torch.einsum("qhd,khd->hqk", q, k) / d ** 0.5
            sc = sc.masked_fill(torch.triu(torch.ones(n, n, dtype=torch.bool), 1), float("-inf"))
            o = torch.einsum("hqk,khd->qhd", sc.softmax(-1), v).reshape(n, nq * d)
            h = h + o @ lw.o.float().cpu().t()
            y = rms(h, lw.ln2.cpu())
            gu = y @ lw.gate_up.float().cpu().t()
            i = gu.shape[1] // 2
            h = h + (torch.nn.functional.silu(gu[:, :i]) * gu[:, i:]) @ lw.down.float().cpu().t()
        y = rms(h[-1:], m.final_ln.cpu())
        outs.append(y @ m.lm_head.float().cpu().t())
    return torch.cat(outs)


LENS = [40, 70, 17]


def _tokens():
    g = torch.Generator().manual_seed(5)
    return torch.randint(0, 1024, (sum(LENS),), generator=g)


def test_tp1_prefill_matches_fp32_reference():
    tokens = _tokens()
    logits, alarms, checks, _, m = _prefill_logits(1, 0, LENS, tokens)
    ref = _reference(m, LENS, tokens)
    err = (logits - ref).abs().max().item()
    assert err < 0.03 * ref.abs().max().item(), (err, ref.abs().max().item())
    assert checks > 0 and not alarms, alarms


def test_tp1_prefill_fused_push_path_matches_fp32_reference():
    """512 tokens: the row-parallel GEMMs take the fused GEMM + reduce-scatter push path."""
    lens = [200, 312]
    g = torch.Generator().manual_seed(6)
    tokens = torch.randint(0, 1024, (sum(lens),), generator=g)
    logits, alarms, checks, _, m = _prefill_logits(1, 0, lens, tokens)
    ref = _reference(m, lens, tokens)
    err = (logits - ref).abs().max().item()
    assert err < 0.03 * ref.abs().max().item(), (err, ref.abs().max().item())
    assert checks > 0 and not alarms, alarms


def test_tp1_injected_transfer_flip_is_reported():
    _, _, _, hit, _ = _prefill_logits(1, 0, LENS, _tokens(), inject=True)
    assert hit and hit[0][0].startswith("reduce_scatter") and hit[0][1] == 0 and hit[0][2] == 0, hit


def _worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
        import datetime
        import torch.distributed as dist
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=60))
        logits, alarms, checks, hit, _ = _prefill_logits(world, rank, LENS, _tokens(), inject=True)
        q.put((rank, logits, len(alarms), checks, hit))
        dist.destroy_process_group()
    except Exception as e:       # reported to the parent
        q.put((rank, repr(e), -1, 0, None))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_matches_tp1():
    import torch.multiprocessing as mp
    ref, _, _, _, _ = _prefill_logits(1, 0, LENS, _tokens())
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = {}
    for _ in ps:
        r = q.get(timeout=240)
        res[r[0]] = r
    for p in ps:
        p.join(timeout=60)
    for r in (0, 1):
        assert not isinstance(res[r][1], str), res[r][1]
        assert res[r][2] == 0 and res[r][3] > 0
    err = (res[0][1] - ref).abs().max().item()
    assert err < 0.02 * ref.abs().max().item(), err
    assert torch.equal(res[0][1], res[1][1])
    # rank 1 flipped a bit of its partial at row 0: rank 0 owns row 0 and must name peer 1
    assert res[0][4] and res[0][4][0][0].startswith("reduce_scatter") and res[0][4][0][3] == 1, res[0][4]
