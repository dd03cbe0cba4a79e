"""A device-side wait that runs out returns an error status and leaves the context usable (no trap, no hang).

The tensor-parallel all-gather waits for every rank's generation flag before it pulls. Here both "ranks" are
buffers on this one GPU and rank 1's flag is never raised, so the single launch's wait runs out after the short
limit set for the test; the kernel records ERR_TIMEOUT_PEER in its error word and returns. Raising the flag and
launching again then completes with the right rows and a clean error word. The checked GEMM's band counters are
zeroed when the error word is taken (`ops.gemm.take_errors`), so the next GEMM starts clean."""
import ctypes
import time

import pytest
import torch

from sdcguard_b200 import _native
from sdcguard_b200.numerics import abft
from sdcguard_b200.ops import gemm

pytestmark = pytest.mark.gpu

ERR_TIMEOUT_PEER = 4


_KEEP = []


def _ptrs(ts):
    """Host table of device pointers, as the launchers take it (kept alive for the test's duration)."""
    arr = (ctypes.c_ulonglong * 8)(*[t.data_ptr() for t in ts], *([0] * (8 - len(ts))))
    _KEEP.append(arr)
    return ctypes.cast(arr, ctypes.c_void_p)


def test_peer_wait_runs_out_and_reports():
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    R, N, world = 128, 256, 2
    nb = N // 128
    g = torch.Generator(device=dev).manual_seed(0)
    shards = [torch.randn(R, N, device=dev, generator=g).bfloat16() for _ in range(world)]
    seals = [torch.empty(R, nb, dtype=torch.int32, device=dev) for _ in range(world)]
    for s, sl in zip(shards, seals):
        _native.check(_native.lib().sdc_seal_rows(s.data_ptr(), N, R, N, sl.data_ptr(),
                                                  torch.cuda.current_stream().cuda_stream), "seal rows")
    gen = torch.ones(1, dtype=torch.int64, device=dev)
    flags = torch.tensor([1, 0], dtype=torch.int64, device=dev)       # rank 1 never signals
    out = torch.zeros(world * R, N, dtype=torch.bfloat16, device=dev)
    state = torch.zeros(1, abft.STATE_COLS, dtype=torch.int64, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    sp, slp = _ptrs(shards), _ptrs(seals)
    _native.set_wait_limit(20_000_000)                                 # 20 ms for this test
    try:
        torch.cuda.synchronize()
        t0 = time.time()
        _native.check(_native.lib().sdc_tp_all_gather(sp, slp, gen.data_ptr(), flags.data_ptr(), world, R, N,
                                                      out.data_ptr(), state.data_ptr(), err.data_ptr(), None, None,
                                                      torch.cuda.current_stream().cuda_stream), "all-gather")
        torch.cuda.synchronize()                    # the launch ends: no hang, no fault
        waited = time.time() - t0
        assert int(err.item()) == ERR_TIMEOUT_PEER
        assert waited < 5.0
        assert int(out.abs().sum().item()) == 0     # nothing was pulled after the wait ran out
        # the context is usable: raise the flag, clear the error word, launch again
        flags[1] = 1
        err.zero_()
        _native.check(_native.lib().sdc_tp_all_gather(sp, slp, gen.data_ptr(), flags.data_ptr(), world, R, N,
                                                      out.data_ptr(), state.data_ptr(), err.data_ptr(), None, None,
                                                      torch.cuda.current_stream().cuda_stream), "all-gather")
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        assert torch.equal(out, torch.cat(shards))
        row = abft.decode_state_row(state[0].tolist())
        assert row["z"] == 0 and row["checks"] >= 1
    finally:
        _native.set_wait_limit()                    # back to the default deadline


def test_taken_error_zeroes_gemm_band_counters():
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    m, n, k = 256, 512, 256
    x = torch.randn(m, k, device=dev).bfloat16()
    w = (torch.randn(n, k, device=dev) * 0.05).bfloat16()
    cw = gemm.CheckedWeight(w)
    table = gemm.StateTable(dev, 2)
    slot = table.add("t (ABFT GEMM)", cw.nb)
    gemm.checked_linear(x, cw, table.state, slot)
    torch.cuda.synchronize()
    ws = gemm.workspace(dev, 0)
    cb = int(_native.lib().sdc_gemm_counter_bytes())
    assert int(ws[:cb].sum().item()) == 0           # a completed launch leaves its counters at zero
    ws[:cb].fill_(7)                                # what a launch stopped mid-band would leave
    gemm.error_word(dev).fill_(ERR_TIMEOUT_PEER)
    assert gemm.take_errors(dev) == ERR_TIMEOUT_PEER
    assert int(ws[:cb].sum().item()) == 0 and gemm.take_errors(dev) == 0
    table.read(reset=True)
    y = gemm.checked_linear(x, cw, table.state, slot)
    torch.cuda.synchronize()
    r = table.read(reset=True)[0]
    assert r["checks"] >= 1 and r["unjudged"] == 0 and r["z"] < abft.Z_ALARM
    ref = (x.float() @ w.float().t())
    assert torch.allclose(y.float(), ref, atol=2e-2, rtol=2e-2)
