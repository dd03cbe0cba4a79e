"""Tensor-parallel collectives with carried checksums: world size 1 in-process (any GPU box) and world size 2 across
processes (skipped with fewer than 2 GPUs). Outputs are compared with plain PyTorch fp32 sums; a flipped bit in a
partial or a shard after it was sealed must be reported at the right rows."""
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


def _partials(world, M, K, H, seed=0):
    g = torch.Generator().manual_seed(seed)
    xs = [torch.randn(M, K, generator=g).bfloat16() for _ in range(world)]
    ws = [(torch.randn(H, K, generator=g) * 0.05).bfloat16() for _ in range(world)]
    return xs, ws


def _rank_body(rank, world, M, K, H, flip):
    from sdcguard_b200.ops import gemm
    from sdcguard_b200.parallel.symm import LocalHeap, SymmetricHeap
    from sdcguard_b200.parallel.tp import TPComm
    dev = torch.device("cuda", rank)
    heap = SymmetricHeap(device=dev) if world > 1 else LocalHeap(dev)
    comm = TPComm(heap, M, H)
    xs, ws = _partials(world, M, K, H)
    x, w = xs[rank].to(dev), ws[rank].to(dev)
    cw = gemm.CheckedWeight(w)
    st = gemm.StateTable(dev, 2)
    sl = st.add("rowpar", cw.nb)
    gemm.checked_linear(x, cw, st.state, sl, out=comm.partial(M), seal=comm.partial_seal(M))
    if flip is not None and rank == flip[0]:
        torch.cuda.synchronize(dev)
        comm.partial(M).view(torch.int16)[flip[1], flip[2]] ^= 1
    R = M // world
    out = torch.empty(R, H, dtype=torch.bfloat16, device=dev)
    comm.reduce_scatter(M, out)
    torch.cuda.synchronize(dev)
    ref = sum(xs[r].float() @ ws[r].float().t() for r in range(world))[rank * R:(rank + 1) * R].to(dev)
    err = (out.float() - ref).abs().max().item()
    rs = comm.read_state()
    # all-gather of this rank's rows of the reduced output
    comm.shard(R).copy_(out)
    full = torch.empty(M, H, dtype=torch.bfloat16, device=dev)
    comm.all_gather(R, full)
    torch.cuda.synchronize(dev)
    ag = comm.read_state()
    mine = torch.equal(full[rank * R:(rank + 1) * R], out)
    comm.close()          # waits for every rank: a peer may still be reading this rank's buffers
    return {"err": err, "scale": ref.abs().max().item(), "rs": rs["reduce_scatter"], "ag": ag["all_gather"],
            "mine": mine, "error": rs["error"], "gemm_z": st.read()[0]["z"]}


def test_world1_collectives_and_seals():
    r = _rank_body(0, 1, 512, 256, 1024, None)
    assert r["err"] <= 2 ** -7 * r["scale"] + 1e-2
    assert r["rs"]["z"] == 0.0 and r["rs"]["checks"] == 1 and r["ag"]["z"] == 0.0 and r["mine"]
    r = _rank_body(0, 1, 512, 256, 1024, (0, 300, 517))
    assert (r["rs"]["flat"] // 8) // 8 == 300 and r["rs"]["z"] == float("inf")


def _worker(rank, world, port, flip, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    import datetime
    torch.distributed.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                                         device_id=torch.device("cuda", rank))
    try:
        q.put((rank, _rank_body(rank, world, 512, 256, 1024, flip)))
    except Exception as e:  # noqa: BLE001  report instead of leaving the parent waiting
        q.put((rank, {"exception": repr(e)}))
        raise
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("flip", [None, (1, 40, 900)])
def test_world2_collectives_over_nvlink(flip):
    ctx = torch.multiprocessing.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, flip, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=150) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        assert res[r]["error"] == 0
        assert res[r]["mine"]
    if flip is None:
        for r in range(2):
            assert res[r]["err"] <= 2 ** -7 * res[r]["scale"] + 1e-2, res
            assert res[r]["rs"]["z"] == 0.0 and res[r]["ag"]["z"] == 0.0
    else:
        # row 40 belongs to rank 0's rows: rank 0 sees peer 1's bad seal; rank 1 sees nothing
        assert res[0]["rs"]["z"] == float("inf") and res[0]["rs"]["flat"] % 8 == 1
        assert res[1]["rs"]["z"] == 0.0
