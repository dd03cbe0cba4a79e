"""Row-parallel checked GEMM fused with the reduce-scatter transfer (push mode): the GEMM epilogue stores every tile
into the owner rank's receive buffer, the owner sums its slots locally. Compared with the two-step path (checked GEMM
into the local partial, then the pull reduce-scatter) and with an fp32 reference; an accumulator flip inside the
GEMM and a bit flip in a received slot are both reported. World 2 runs as two processes (skipped with fewer GPUs)."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

M, K, N = 512, 2048, 1024


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _data(world):
    g = torch.Generator().manual_seed(11)
    x = torch.randn(world, M, K, generator=g).mul(0.5)
    w = torch.randn(world, N, K, generator=g).mul(K ** -0.5)
    return x.bfloat16(), w.bfloat16()


def _run(world, rank):
    from sdcguard_b200.ops import gemm
    from sdcguard_b200.parallel.symm import LocalHeap, SymmetricHeap
    from sdcguard_b200.parallel.tp import TPComm
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    heap = SymmetricHeap(device=dev) if world > 1 else LocalHeap(dev)
    comm = TPComm(heap, M, N)
    xs, ws = _data(world)
    x, w = xs[rank].to(dev), ws[rank].to(dev)
    cw = gemm.CheckedWeight(w)
    st = gemm.StateTable(dev)
    slot = st.add("rowpar", cw.nb)
    R = M // world
    res = {}
    # two-step path: checked GEMM with seals into the local partial, then the pull reduce-scatter
    gemm.checked_linear(x, cw, st.state, slot, out=comm.partial(M), seal=comm.partial_seal(M))
    pull = comm.reduce_scatter(M, torch.empty(R, N, dtype=torch.bfloat16, device=dev))
    # fused path
    push = comm.gemm_reduce_scatter(x, cw, st.state, slot, torch.empty(R, N, dtype=torch.bfloat16, device=dev))
    torch.cuda.synchronize(dev)
    res["pull"], res["push"] = pull.float().cpu(), push.float().cpu()
    res["clean_gemm"] = [r for r in st.read(reset=True) if r["z"] > 6]
    cs = comm.read_state()
    res["clean_comm"] = (cs["reduce_scatter"]["z"], cs["error"], cs["reduce_scatter"]["checks"])
    # an accumulator flip inside the fused GEMM (rank 0, row R + 3 belongs to rank 1 when world is 2)
    inj_row = min(R + 3, M - 1)
    for _ in range(2):   # repeat: the second launch reuses the flags / done counter of the first
        comm.gemm_reduce_scatter(x, cw, st.state, slot, torch.empty(R, N, dtype=torch.bfloat16, device=dev),
                                 inject=(inj_row, 77, 1 << 28) if rank == 0 else None)
    torch.cuda.synchronize(dev)
    res["gemm_hit"] = [(r["row"], r["block"]) for r in st.read(reset=True) if r["z"] > 6]
    comm.read_state()
    # a flip in this rank's own received slot (its own tile, so it has landed when the stream is synchronised)
    comm.inject_next(rank * R + 5, 130, 6)
    comm.gemm_reduce_scatter(x, cw, st.state, slot, torch.empty(R, N, dtype=torch.bfloat16, device=dev))
    torch.cuda.synchronize(dev)
    cs = comm.read_state()
    loc = None
    if cs["reduce_scatter"]["z"] > 6:
        rb, peer = divmod(cs["reduce_scatter"]["flat"], 8)
        loc = (*divmod(rb, comm.nb), peer)
    res["xfer_hit"] = loc
    comm.close()
    return res


def _check(res, world, rank):
    xs, ws = _data(world)
    R = M // world
    ref = sum(xs[r].float() @ ws[r].float().t() for r in range(world))[rank * R:(rank + 1) * R]
    assert torch.equal(res["push"], res["pull"])
    err = (res["push"] - ref).abs().max().item()
    assert err < 0.02 * ref.abs().max().item(), err
    assert not res["clean_gemm"], res["clean_gemm"]
    z, e, checks = res["clean_comm"]
    assert z <= 6 and e == 0 and checks > 0, res["clean_comm"]
    assert res["xfer_hit"] == (5, 1, rank), res["xfer_hit"]


def test_push_world1():
    res = _run(1, 0)
    _check(res, 1, 0)
    assert res["gemm_hit"] == [(min(M // 1 + 3, M - 1), 0)], res["gemm_hit"]


def _worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
        import datetime
        import torch.distributed as dist
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=60))
        q.put((rank, _run(world, rank)))
        dist.destroy_process_group()
    except Exception as e:       # reported to the parent
        q.put((rank, repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_push_world2():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = {}
    for _ in ps:
        r, v = q.get(timeout=240)
        res[r] = v
    for p in ps:
        p.join(timeout=60)
    for r in (0, 1):
        assert not isinstance(res[r], str), res[r]
        _check(res[r], 2, r)
    # rank 0 flipped an accumulator of row R + 3, a row rank 1 owns; the GEMM check runs on rank 0
    assert res[0]["gemm_hit"] == [(M // 2 + 3, 0)], res[0]["gemm_hit"]
    assert not res[1]["gemm_hit"], res[1]["gemm_hit"]
