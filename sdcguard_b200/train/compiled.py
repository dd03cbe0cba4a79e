"""Protected layers inside torch.compile (fullgraph included) and under DTensor tensor parallelism.

Under compilation a protected layer's forward is one custom operator, `sdcguard_b200::checked_linear`, which the
compiler keeps as an opaque call; its backward is a second operator, `sdcguard_b200::checked_linear_backward`. At
run time they run the same checked GEMMs as eager mode (the tcgen05 kernel with the ABFT check of its fp32
accumulator, for the forward, dX and dW) when the guard is active, and plain PyTorch otherwise. The guard's
`active` flag is read while tracing, so a checked and an unchecked graph are each compiled once: unchecked steps
run the plain, fully optimized graph.

Both operators are tagged `cudagraph_unsafe`: under mode="reduce-overhead" Inductor runs them outside its CUDA
graphs, so their checks run on every checked step (inside a replayed graph an operator's Python would not run and
its checks would silently stop).

Tensor parallel: both operators have DTensor sharding rules, so DTensor calls them on each rank's local shards and
each rank checks its own GEMM: replicated, batch or sequence sharded inputs, column parallel (weight and bias
sharded by output features) and row parallel (input sharded by its last dimension, weight by input features: the
output is a partial sum, checked before DTensor's reduction). These are the layouts ColwiseParallel and
RowwiseParallel produce, so DTensor adds no communication; another layout is redistributed to one of them first.

Reference: src/sdcguard/_compiled.py:44-155 (the same two-operator structure and rule set: PyTorch's custom
operator and DTensor APIs dictate it).
"""
from __future__ import annotations

import itertools
import weakref
from typing import Optional

import torch
import torch.nn.functional as F

_STATES: "weakref.WeakValueDictionary" = weakref.WeakValueDictionary()
_IDS = itertools.count(1)
_TAGS = tuple(t for t in (getattr(torch.Tag, "cudagraph_unsafe", None),) if t is not None)


def register(state) -> int:
    """An id the operators use to find a protected layer's guard state (kept weakly)."""
    i = next(_IDS)
    _STATES[i] = state
    return i


def _fresh(t: torch.Tensor) -> torch.Tensor:
    return t if t._base is None else t.clone()       # a custom operator's output cannot alias its input


@torch.library.custom_op("sdcguard_b200::checked_linear", mutates_args=(), tags=_TAGS)
def checked_linear(x: torch.Tensor, w: torch.Tensor, b: Optional[torch.Tensor], state_id: int) -> torch.Tensor:
    st = _STATES.get(state_id)
    with torch.autocast(device_type=x.device.type, enabled=False):
        if st is None or not st.runnable(x, w):
            return F.linear(x, w, b)
        return _fresh(st.checked_forward(x, w, b))


@checked_linear.register_fake
def _(x, w, b, state_id):
    return x.new_empty((*x.shape[:-1], w.shape[0]))


@torch.library.custom_op("sdcguard_b200::checked_linear_backward", mutates_args=(), tags=_TAGS)
def checked_linear_backward(gy: torch.Tensor, x: torch.Tensor, w: torch.Tensor, state_id: int, need_x: bool,
                            need_w: bool, need_b: bool) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    st = _STATES.get(state_id)
    with torch.autocast(device_type=gy.device.type, enabled=False):
        if st is None or not st.runnable(x, w):
            g2 = gy.reshape(-1, gy.shape[-1])
            gx = g2.mm(w.to(g2.dtype)).view(x.shape).to(x.dtype) if need_x else None
            gw = g2.t().mm(x.reshape(-1, x.shape[-1]).to(g2.dtype)).to(w.dtype) if need_w else None
            gb = g2.float().sum(0).to(w.dtype) if need_b else None
        else:
            gx, gw, gb = st.checked_backward(gy, x, w, need_x, need_w, need_b)
    return tuple(gy.new_empty(0) if t is None else _fresh(t) for t in (gx, gw, gb))


@checked_linear_backward.register_fake
def _(gy, x, w, state_id, need_x, need_w, need_b):
    return (x.new_empty(x.shape) if need_x else gy.new_empty(0),
            w.new_empty(w.shape) if need_w else gy.new_empty(0),
            w.new_empty(w.shape[0]) if need_b else gy.new_empty(0))


def _setup(ctx, inputs, output):
    x, w, b, state_id = inputs
    ctx.save_for_backward(x, w)
    ctx.has_bias = b is not None
    ctx.state_id = state_id


def _backward(ctx, gy):
    x, w = ctx.saved_tensors
    nx, nw, nb = ctx.needs_input_grad[:3]
    nb = bool(nb and ctx.has_bias)
    gx, gw, gb = checked_linear_backward(gy, x, w, ctx.state_id, bool(nx), bool(nw), nb)
    return gx if nx else None, gw if nw else None, gb if nb else None, None


checked_linear.register_autograd(_backward, setup_context=_setup)


def _sharding_rules() -> bool:
    """DTensor rules for both operators, per mesh dimension. False when this PyTorch has no DTensor API."""
    try:
        from torch.distributed.tensor import Partial, Replicate, Shard
        from torch.distributed.tensor.experimental import register_sharding
    except Exception:  # noqa: BLE001  (a build without distributed, or without the API)
        return False
    R = Replicate()

    def fwd(x, w, b, state_id):
        last = x.ndim - 1
        bb = (lambda p: None) if b is None else (lambda p: p)
        rules = [([R], [R, R, bb(R), None])]
        rules += [([Shard(d)], [Shard(d), R, bb(R), None]) for d in range(last)]          # batch / sequence
        rules.append(([Shard(last)], [R, Shard(0), bb(Shard(0)), None]))                   # column parallel
        rules.append(([Partial()], [Shard(last), Shard(1), bb(Partial()), None]))          # row parallel
        rules.append(([Partial()], [Partial(), R, bb(Partial()), None]))                   # a partial input
        return rules

    def bwd(gy, x, w, state_id, need_x, need_w, need_b):
        last = gy.ndim - 1

        def out(gx, gw, gb):
            return [gx if need_x else R, gw if need_w else R, gb if need_b else R]
        tail = [None] * 4
        rules = [(out(R, R, R), [R, R, R] + tail)]
        rules += [(out(Shard(d), Partial(), Partial()), [Shard(d), Shard(d), R] + tail) for d in range(last)]
        rules.append((out(Partial(), Shard(0), Shard(0)), [Shard(last), R, Shard(0)] + tail))   # column parallel
        rules.append((out(Shard(last), Shard(1), R), [R, Shard(last), Shard(1)] + tail))        # row parallel
        rules.append((out(R, Partial(), R), [R, Partial(), R] + tail))                          # a partial input
        return rules

    try:
        register_sharding(torch.ops.sdcguard_b200.checked_linear.default)(fwd)
        register_sharding(torch.ops.sdcguard_b200.checked_linear_backward.default)(bwd)
    except Exception:  # noqa: BLE001
        return False
    return True


TENSOR_PARALLEL = _sharding_rules()
