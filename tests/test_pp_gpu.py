"""Pipeline parallelism: the decoder split into stages gives the same logits as the whole model (one GPU, stages run
in turn); two processes on two GPUs with sealed NCCL transfers give the same logits again, and a bit flipped in
transit is reported by the receiving stage (skipped with fewer than 2 GPUs)."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

LENS = [40, 70]


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _metas(dev, group):
    from sdcguard_b200.models.decoder import StepMeta
    from sdcguard_b200.ops import attention
    g = torch.Generator().manual_seed(5)
    metas = []
    for mb, n in enumerate(LENS):           # one request per microbatch, pages 1 + 8 mb ...
        pages = list(range(1 + 8 * mb, 1 + 8 * (mb + 1)))
        metas.append(StepMeta(mode="prefill", tokens=torch.randint(0, 1024, (n,), generator=g).to(dev),
                              pos=torch.arange(n, dtype=torch.int32, device=dev),
                              slots=torch.tensor([pages[p // 16] * 16 + p % 16 for p in range(n)], dtype=torch.int64,
                                                 device=dev),
                              block_table=torch.tensor([pages], dtype=torch.int32, device=dev),
                              logits_rows=torch.tensor([n - 1], dtype=torch.int64, device=dev),
                              tiles=attention.prefill_tiles([0], [n], group).to(dev)))
    return metas


def _model(dev):
    from sdcguard_b200.models.decoder import TINY, CheckedDecoder
    m = CheckedDecoder(TINY, dev, checked=True, seed=3)
    m.buffers(256)
    return m


def _cache(m, layers, dev):
    return torch.zeros(layers, 1 + 8 * len(LENS), 2, m.nkv, 16, 128, dtype=torch.bfloat16, device=dev)


def test_staged_forward_matches_whole_model():
    dev = torch.device("cuda:0")
    m = _model(dev)
    metas = _metas(dev, m.nq // m.nkv)
    whole = [m.forward(mt, _cache(m, 2, dev)).float().cpu() for mt in metas]
    staged = []
    for mt in metas:
        c0, c1 = _cache(m, 1, dev), _cache(m, 1, dev)
        x, r = m.forward(mt, c0, layer_range=(0, 1), last=False)
        staged.append(m.forward(mt, c1, layer_range=(1, 2), hidden=(x.clone(), r.clone())).float().cpu())
    for a, b in zip(whole, staged):
        assert torch.equal(a, b)
    assert not [r for r in m.read_checks(reset=True) if r["z"] > 6]


def _worker(rank, port, q, inject):
    try:
        import datetime

        import torch.distributed as dist

        from sdcguard_b200.parallel.pp import SealedP2P, run_stage
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=2, device_id=dev,
                                timeout=datetime.timedelta(seconds=60))
        m = _model(dev)
        comm = SealedP2P(rank, 2, dev)
        if inject and rank == 0:
            comm.inject_next(5, 200, 4)
        outs = run_stage(m, comm, _metas(dev, m.nq // m.nkv), _cache(m, 1, dev))
        torch.cuda.synchronize(dev)
        q.put((rank, [o.float().cpu() for o in outs], comm.read_state(), len([r for r in m.read_checks(reset=True)
                                                                             if r["z"] > 6])))
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e), None, -1))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("inject", [False, True])
def test_pp2_sealed_transfers(inject):
    import torch.multiprocessing as mp
    dev = torch.device("cuda:0")
    m = _model(dev)
    whole = [m.forward(mt, _cache(m, 2, dev)).float().cpu() for mt in _metas(dev, m.nq // m.nkv)]
    del m
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, port, q, inject)) for r in range(2)]
    for p in ps:
        p.start()
    res = {}
    for _ in ps:
        r = q.get(timeout=240)
        res[r[0]] = r
    for p in ps:
        p.join(timeout=60)
    assert not isinstance(res[1][1], str), res[1][1]
    assert res[0][3] == 0 and res[1][3] == 0
    st = res[1][2]
    if inject:
        assert st["z"] == float("inf") and (st["row"], st["block"], st["peer"]) == (5, 1, 0), st
    else:
        assert st["z"] == 0 and st["checks"] == 2 * len(LENS), st
        for a, b in zip(whole, res[1][1]):
            assert torch.equal(a, b)
