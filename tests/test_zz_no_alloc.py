"""The allocation-free checked GEMM entry point (csrc/gemm_noalloc.h), called through its exported C symbol.

It is for callers that cannot allocate GPU memory at call time (allocator callbacks, plugins handed
pre-allocated buffers, paths that must not hit a first-time cudaMalloc). Its output and check results must
match the regular entry point, which takes a caller workspace, on two calls in a row (the shared fixed
workspace keeps the previous call's contents, so the second call exercises that). This file is collected last.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _noalloc_fn():
    from sdcguard_b200 import _native
    _native.lib()                                     # builds the library if needed
    h = ctypes.CDLL(str(_native.LIB_PATH))
    fn = h.sdc_gemm_bf16_noalloc
    P, I, L, U, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong, ctypes.c_uint, ctypes.c_float
    fn.restype = I
    fn.argtypes = [P, L, P, P, I, I, I, P, L, P, P, F, P, P, P, I, U, U, U, U, F, F, F, F, F, P, I, I, P]
    return fn


def _call(fn, x, cw, out, state, slot, row_sq, err):
    import math
    from sdcguard_b200.numerics import abft
    s = cw.mask
    return fn(x.data_ptr(), x.stride(0), cw.weight.data_ptr(), cw.cs.wc.data_ptr(), x.shape[0], cw.n, cw.k,
              out.data_ptr(), out.stride(0), None, None, 0.0, row_sq.data_ptr(), cw.cs.wstat.data_ptr(),
              state.data_ptr(), slot, s[0], s[1], s[2], s[3], abft.Z_ALARM, cw.prod_coef, cw.out_coef,
              abft.ABS_FLOOR, math.sqrt(cw.k), err.data_ptr(), 256, 0,
              torch.cuda.current_stream().cuda_stream)


def test_noalloc_entry_matches_regular_entry_twice():
    from sdcguard_b200.ops import gemm
    fn = _noalloc_fn()
    dev = torch.device("cuda")
    torch.manual_seed(7)
    shapes = [(1000, 3072, 1024), (256, 4096, 1024)]       # the second call sees the first call's leftovers
    for (m, n, k) in shapes:
        x = torch.randn(m, k, device=dev).bfloat16()
        w = (torch.randn(n, k, device=dev) * 0.02).bfloat16()
        cw = gemm.CheckedWeight(w)
        rs = gemm.row_sqnorm(x)
        st = gemm.StateTable(dev, 4)
        a, b = st.add("regular", cw.nb), st.add("noalloc", cw.nb)
        # the regular entry splits K for decode-sized M; the allocation-free one never does: compare with the
        # regular entry's one-pass kernel (a CTA cap turns the split off)
        nsm = torch.cuda.get_device_properties(dev).multi_processor_count
        y_ref = gemm.checked_linear(x, cw, st.state, a, row_sq=rs, bn=256, max_ctas=nsm)
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        y = torch.empty_like(y_ref)
        assert _call(fn, x, cw, y, st.state, b, rs, err) == 0
        torch.cuda.synchronize()
        ref32 = x.float() @ w.float().t()
        assert (y.float() - ref32).abs().max().item() <= 2 ** -7 * ref32.abs().max().item() + 1e-3
        assert torch.equal(y, y_ref)
        r = st.read()
        assert r[b]["checks"] == 1 and r[b]["unjudged"] == 0
        assert abs(r[b]["z"] - r[a]["z"]) <= 1e-6 * max(1.0, r[a]["z"]) and r[b]["z"] < 2.0
        assert err.item() == 0


def test_noalloc_rejects_too_large_problem():
    from sdcguard_b200.ops import gemm
    fn = _noalloc_fn()
    dev = torch.device("cuda")
    x = torch.zeros(8192, 64, device=dev, dtype=torch.bfloat16)
    cw = gemm.CheckedWeight(torch.zeros(65536, 64, device=dev, dtype=torch.bfloat16))
    out = torch.empty(8192, 65536, device=dev, dtype=torch.bfloat16)
    st = torch.zeros(1, 4, dtype=torch.int64, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    rs = torch.zeros(8192, device=dev)
    assert _call(fn, x, cw, out, st, 0, rs, err) == -10
