"""The protected layer's custom operators for torch.compile: registration consistency (opcheck: schema, fake
kernel, autograd), a fullgraph compile of a protected model, and the DTensor sharding rules on two gloo ranks
(column and row parallel give the unsharded layer's output and gradients)."""
import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from sdcguard_b200.train import compiled


def test_opcheck_and_unregistered_state():
    x = torch.randn(4, 16, requires_grad=True)
    w = torch.randn(8, 16, requires_grad=True)
    b = torch.randn(8, requires_grad=True)
    torch.library.opcheck(torch.ops.sdcguard_b200.checked_linear.default, (x, w, b, 0))
    y = compiled.checked_linear(x, w, b, 0)                    # no state with id 0: plain linear
    assert torch.allclose(y, torch.nn.functional.linear(x, w, b))
    y.sum().backward()
    assert torch.allclose(w.grad, torch.ones(4, 8).t() @ x.detach())
    assert torch.allclose(b.grad, torch.full((8,), 4.0))


def test_fullgraph_compile_of_protected_model():
    from sdcguard_b200.train.guard import SDCGuard
    torch.manual_seed(0)
    m = torch.nn.Sequential(torch.nn.Linear(16, 32), torch.nn.ReLU(), torch.nn.Linear(32, 8))
    ref = torch.nn.Sequential(torch.nn.Linear(16, 32), torch.nn.ReLU(), torch.nn.Linear(32, 8))
    ref.load_state_dict(m.state_dict())
    g = SDCGuard(check_every=1, device="cpu")
    g.protect(m)
    cm = torch.compile(m, backend="aot_eager", fullgraph=True)
    x = torch.randn(4, 16)
    with g.on_step(0):
        y = cm(x)
    y2 = cm(x)                                                  # the unchecked graph
    assert torch.allclose(y, ref(x), atol=1e-6) and torch.allclose(y2, ref(x), atol=1e-6)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _tp_worker(rank, world, port, q):
    try:
        import torch.distributed as dist
        from torch.distributed.device_mesh import init_device_mesh
        from torch.distributed.tensor import Replicate, Shard, distribute_tensor
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
        mesh = init_device_mesh("cpu", (world,))
        torch.manual_seed(0)
        x = torch.randn(6, 16)
        w = torch.randn(8, 16)
        b = torch.randn(8)
        full = torch.nn.functional.linear(x, w, b)
        # column parallel: weight and bias sharded by output features
        xd = distribute_tensor(x, mesh, [Replicate()])
        wd = distribute_tensor(w, mesh, [Shard(0)])
        bd = distribute_tensor(b, mesh, [Shard(0)])
        col = compiled.checked_linear(xd, wd, bd, 0)
        ok_col = torch.allclose(col.full_tensor(), full, atol=1e-5) and col.placements[0] == Shard(1)
        # row parallel: input by its last dimension, weight by input features; bias replicated
        xr = distribute_tensor(x, mesh, [Shard(1)])
        wr = distribute_tensor(w, mesh, [Shard(1)])
        br = distribute_tensor(b, mesh, [Replicate()])
        row = compiled.checked_linear(xr, wr, br, 0)
        ok_row = torch.allclose(row.full_tensor(), full, atol=1e-5)
        # gradients through the backward operator (column parallel)
        wg = distribute_tensor(w, mesh, [Shard(0)]).requires_grad_()
        out = compiled.checked_linear(xd, wg, bd, 0)
        out.sum().backward()
        ok_grad = torch.allclose(wg.grad.full_tensor(), torch.ones(6, 8).t() @ x, atol=1e-5)
        q.put((rank, {"col": ok_col, "row": ok_row, "grad": ok_grad, "rules": compiled.TENSOR_PARALLEL}))
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001  (reported to the parent)
        q.put((rank, repr(e)))


def test_dtensor_rules_two_ranks():
    if not compiled.TENSOR_PARALLEL:
        pytest.skip("this PyTorch has no DTensor sharding-rule API")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_tp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=180) for _ in ps)
    for p in ps:
        p.join(timeout=60)
    for r in (0, 1):
        assert isinstance(res[r], dict), res[r]
        assert res[r] == {"col": True, "row": True, "grad": True, "rules": True}, res[r]
