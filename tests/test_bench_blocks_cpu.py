"""bench.py's multi-GPU blocks run as jobs of their own: every rank starts one process of the block's module in a
torch.distributed world of its own, the ranks agree on the outcome, and a block that fails on one rank or hangs
past its limit ends with an error on every rank (the headline measured before it stands). Two gloo ranks on the
CPU, with stand-in block modules."""
import json
import os
import sys
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = '''
import json, os, sys, time
mode = sys.argv[1]
rank = int(os.environ["RANK"])
if mode == "fail" and rank == 1:
    sys.exit(3)
if mode == "hang":
    time.sleep(120)
import torch.distributed as dist
dist.init_process_group("gloo")
t = __import__("torch").tensor([rank + 1.0])
dist.all_reduce(t)
env = {k: os.environ.get(k) for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "MASTER_ADDR", "MASTER_PORT",
                                       "NCCL_NVLS_ENABLE")}
env["elastic"] = sorted(k for k in os.environ if k.startswith("TORCHELASTIC_"))
if rank == 0:
    print("noise")
    print(json.dumps({"sum": float(t.item()), "env": env}))
dist.destroy_process_group()
'''


def _rank(rank, world, port, moddir, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      TORCHELASTIC_RUN_ID="stand-in", SDCGUARD_BLOCK_LOG_DIR=str(moddir),
                      PYTHONPATH=str(moddir) + os.pathsep + os.environ.get("PYTHONPATH", ""))
    sys.path.insert(0, ROOT)
    import bench
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import argparse
    out = {"left": bench.time_left(argparse.Namespace(deadline=1000.0))}
    for mode, limit in (("ok", 120.0), ("fail", 15.0), ("hang", 4.0)):
        t0 = time.perf_counter()
        r = bench.run_child_block(mode, "sdc_block_child", [mode], rank, world, rank, limit)
        out[mode] = (r, time.perf_counter() - t0)
    dist.destroy_process_group()
    q.put((rank, out))


def test_child_blocks_agree_and_fail_cleanly(tmp_path):
    (tmp_path / "sdc_block_child.py").write_text(CHILD)
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, tmp_path, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # the deadline as rank 0 sees it, the same on every rank
    assert got[0]["left"] == got[1]["left"] and 0 < got[0]["left"] <= 1000.0
    ok0, ok1 = got[0]["ok"][0], got[1]["ok"][0]
    assert ok0["sum"] == 3.0 and ok1 == {}, got
    env = ok0["env"]
    assert env["RANK"] == "0" and env["WORLD_SIZE"] == "2" and env["MASTER_ADDR"] == "127.0.0.1"
    assert env["MASTER_PORT"] != str(port) and env["NCCL_NVLS_ENABLE"] == "0" and env["elastic"] == []
    assert ok0["block_wall_s"] >= 0
    # a process that fails on one rank: both ranks report an error, the failing one names its exit code
    f0, f1 = got[0]["fail"][0], got[1]["fail"][0]
    assert "error" in f0 and "error" in f1 and "rc 3" in f1["error"], got
    # a process that hangs past the limit is ended; the block returns within a few seconds of it
    (h0, t0), (h1, t1) = got[0]["hang"], got[1]["hang"]
    assert "error" in h0 and "error" in h1 and t0 < 60 and t1 < 60, got
