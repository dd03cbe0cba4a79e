"""Sealed pipeline transfers between two gloo ranks on the CPU: a clean transfer verifies, a bit flipped after
sealing is reported with its row, block and sending stage; the layer split."""
import os
import socket

import torch
import torch.multiprocessing as mp

from sdcguard_b200.parallel.pp import stage_layers


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, port, q):
    import torch.distributed as dist

    from sdcguard_b200.parallel.pp import SealedP2P
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2)
    try:
        comm = SealedP2P(rank, 2, "cpu")
        g = torch.Generator().manual_seed(1)
        x = torch.randn(40, 300, generator=g).bfloat16()
        r = torch.randn(40, 300, generator=g).bfloat16()
        res = []
        for inject in (False, True):
            if rank == 0:
                if inject:
                    comm.inject_next(17, 260, 5)
                for w in comm.send([x, r], 1):
                    if hasattr(w, "wait"):
                        w.wait()
            else:
                got = comm.recv([(40, 300), (40, 300)], 0)
                res.append((bool(torch.equal(got[1], r)), comm.read_state()))
        q.put((rank, res))
    finally:
        dist.destroy_process_group()


def test_sealed_p2p_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
    (same0, clean), (same1, hit) = out[1]
    assert same0 and same1 and clean["z"] == 0 and clean["checks"] == 2
    assert hit["z"] == float("inf") and (hit["row"], hit["block"], hit["peer"]) == (17, 2, 0), hit


def test_stage_layers_split():
    assert [stage_layers(32, s, 4) for s in range(4)] == [(0, 8), (8, 16), (16, 24), (24, 32)]
    assert [stage_layers(28, s, 3) for s in range(3)] == [(0, 10), (10, 19), (19, 28)]
