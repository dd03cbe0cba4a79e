"""Data-parallel majority votes on CPU (gloo, 3 ranks): the canary finds the rank whose layer output differs from
the others' for the same batch, and the replica check finds the rank whose weights differ after a step."""
import os
import socket

import torch
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _body(rank, world, port, q):
    try:
        import datetime
        import torch.distributed as dist
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        from sdcguard_b200.train.canary import Canary
        from sdcguard_b200.train.replica import check_replicas
        torch.manual_seed(0)
        model = torch.nn.Sequential(torch.nn.Linear(16, 32), torch.nn.ReLU(), torch.nn.Linear(32, 4))
        x = torch.randn(8, 16)
        if rank == 2:          # a fault in rank 2's second linear layer output
            model[2].register_forward_hook(lambda m, i, o: o.index_fill_(0, torch.tensor([3]), 7.0))
        can = Canary(model)
        with can.recording():
            model(x)
        ev = can.check(step=5)
        clean_rep = check_replicas(model.parameters(), step=5)
        if rank == 1:
            with torch.no_grad():
                model[0].weight.view(-1)[9] += 1e-3
        bad_rep = check_replicas(model.parameters(), step=6)
        q.put((rank, [e.detail for e in ev], len(clean_rep), [e.detail for e in bad_rep]))
        dist.destroy_process_group()
    except Exception as e:      # reported to the parent
        q.put((rank, repr(e), None, None))


def test_canary_and_replica_votes_find_the_odd_rank():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_body, args=(r, 3, port, q)) for r in range(3)]
    for p in ps:
        p.start()
    res = {}
    for _ in ps:
        r = q.get(timeout=120)
        res[r[0]] = r
    for p in ps:
        p.join(timeout=30)
    for r in range(3):
        assert not isinstance(res[r][1], str), res[r][1]
        can, clean, bad = res[r][1], res[r][2], res[r][3]
        assert len(can) == 1 and can[0]["suspect_ranks"] == [2] and can[0]["call"] == 2
        assert clean == 0
        assert len(bad) == 1 and bad[0]["suspect_ranks"] == [1]
        # the suspects' identities were gathered; one rank (the lowest that agreed with the majority) reports
        assert can[0]["suspects"][0]["rank"] == 2 and can[0]["suspects"][0]["host"] and can[0]["clear_majority"]
        assert can[0]["reported_by_rank"] == r and can[0]["reporter"] == (r == 0)
        assert bad[0]["reporter"] == (r == 0) and bad[0]["suspect_group_ranks"] == [1]


def test_suspect_event_names_the_suspect_gpu():
    """Built alike on every rank: a single suspect with a clear majority gives the event its GPU's identity; the
    lowest-ranked rank of the majority reports; without a majority rank 0 does."""
    from sdcguard_b200.utils.events import suspect_event
    ids = [{"host": "h", "gpu_uuid": f"GPU-{r}", "pci_bus_id": f"0000:{r:02X}:00.0"} for r in range(4)]
    evs = [suspect_event("canary", 7, [0], ids, me, {"call": 3}, to_job_rank=lambda r: r + 4) for me in range(4)]
    assert all(e.identity["gpu_uuid"] == "GPU-0" for e in evs)
    assert [e.detail["reporter"] for e in evs] == [False, True, False, False]
    assert evs[2].detail["suspect_ranks"] == [4] and evs[2].detail["suspect_group_ranks"] == [0]
    assert evs[2].detail["reported_by_rank"] == 6 and evs[2].detail["suspects"][0]["pci_bus_id"] == "0000:00:00.0"
    split = [suspect_event("replica", 1, [0, 1, 2, 3], ids, me, {}) for me in range(4)]
    assert [e.detail["reporter"] for e in split] == [True, False, False, False]
    assert not split[0].detail["clear_majority"] and split[1].identity["gpu_uuid"] == "GPU-1"
