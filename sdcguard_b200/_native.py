"""Loads the native library (`_lib/libsdcguard_b200.so`, built by `sdcguard_b200._build`) with ctypes and
declares the C signature of every entry point.

The kernels take raw device pointers and a CUDA stream handle; the Python wrappers in `sdcguard_b200.ops`
pass `tensor.data_ptr()` and `torch.cuda.current_stream().cuda_stream`. On a machine with a GPU a missing
or stale library is an error, never a silent fallback: `lib()` builds it when nvcc is available and raises
otherwise.
"""
from __future__ import annotations

import ctypes
import os
import threading
from ctypes import c_float, c_int, c_longlong, c_uint, c_void_p
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "_lib" / "libsdcguard_b200.so"

_lock = threading.Lock()
_lib = None
_launches = [0]            # kernel launches issued through this module since the last reset


class _Counted:
    """Wraps a ctypes function and counts its calls (each entry point below launches one kernel, except the
    size queries)."""

    def __init__(self, fn):
        self._fn = fn

    def __call__(self, *a):
        _launches[0] += 1
        return self._fn(*a)


class _Lib:
    def __init__(self, handle):
        self._h = handle

    def __getattr__(self, name):
        return getattr(self._h, name)


def launch_count() -> int:
    return _launches[0]


def reset_launch_count() -> None:
    _launches[0] = 0

P = c_void_p
I = c_int
L = c_longlong
U = c_uint
U64 = ctypes.c_ulonglong
F = c_float

# name -> (restype, argtypes)
SIGNATURES: dict[str, tuple] = {
    "sdc_gemm_ws_bytes": (L, [I, I]),
    "sdc_gemm_choose_split": (I, [I, I, I, I, I]),
    "sdc_gemm_counter_bytes": (L, []),
    "sdc_gemm_set_capture": (I, [P]),
    "sdc_gemm_capture_bytes": (L, []),
    "sdc_gemm_capture_max_k": (I, []),
    "sdc_gemm_bf16": (I, [P, L, P, P, I, I, I, P, L, P, P, F, P, P, P, P, I, U, U, U, U, F, F, F, F, F, P, I, I, I, I,
                          U, P, P, P]),
    "sdc_row_sqnorm_bf16": (I, [P, L, I, I, P, P]),
    "sdc_add_rmsnorm_bf16": (I, [P, P, P, F, I, I, P, P, P, P, P, P]),
    "sdc_qk_norm_rope_kv": (I, [P, L, I, I, I, I, P, P, P, P, F, P, P, P, P, P, P]),
    "sdc_silu_mul_bf16": (I, [P, I, I, P, P, P, P, P]),
    "sdc_compare_rows_bf16": (I, [P, L, P, P, L, I, I, P, P]),
    "sdc_attn_prefill": (I, [P, P, P, L, P, I, P, P, I, P, I, I, I, F, P, P, P]),
    "sdc_attn_decode": (I, [P, P, P, L, P, I, P, P, P, I, I, I, I, I, F, P, P, P, P]),
    "sdc_gemm_pair_clusters": (I, []),
    "sdc_attn_decode_splits": (I, [I]),
    "sdc_fingerprint_many": (I, [P, I, L, U64, P, P]),
    "sdc_gemm_bf16_push": (I, [P, L, P, P, I, I, I, P, P, F, P, P, P, P, I, U, U, U, U, F, F, F, F, F, P, I, I, I, U,
                               I, I, L, P, P, P, P, P, P]),
    "sdc_tp_reduce_local": (I, [P, P, P, P, I, I, I, I, L, P, F, P, P, P]),
    "sdc_seal_verify": (I, [P, L, I, I, P, I, P, P]),
    "sdc_screen_fma": (I, [L, U64, I, L, P, P]),
    "sdc_screen_special": (I, [L, U64, L, P, P, P]),
    "sdc_screen_compare": (I, [L, P, P, P, P, L, P, P]),
    "sdc_screen_mem_fill": (I, [P, L, L, U64, I, P]),
    "sdc_screen_mem_check": (I, [P, L, L, U64, I, L, P, P]),
    "sdc_gemm_fp8": (I, [P, P, P, P, P, I, I, I, P, L, P, P, P, I, U, U, U, U, F, F, F, F, F, P, I, I, U, P]),
    "sdc_fp8_quant_act": (I, [P, L, I, I, P, P, P, P, P, I, P, P]),
    "sdc_ep_dispatch": (I, [P, P, I, I, I, I, I, I, I, P, P, P, P, P, P, P, P, I, I, I, P]),
    "sdc_ep_receive": (I, [P, P, P, P, P, I, I, I, I, I, P, P, P, P, P, P]),
    "sdc_ep_combine_push": (I, [P, P, P, I, I, I, I, I, I, P, P, P, P, I, I, I, P]),
    "sdc_ep_combine": (I, [P, P, P, P, P, P, I, I, I, I, I, I, I, P, P, P, P]),
    "sdc_router_topk": (I, [P, I, I, I, I, P, P, P, I, P, P]),
    "sdc_tp_signal": (I, [P, P, I, I, P]),
    "sdc_tp_reduce_scatter": (I, [P, P, P, P, I, I, I, I, P, F, P, P, P]),
    "sdc_tp_all_gather": (I, [P, P, P, P, I, I, I, P, P, P, P, P, P]),
    "sdc_add_rmsnorm_shard": (I, [P, P, P, F, I, I, P, P, P, P, I, I, P, P, P, P]),
    "sdc_seal_rows": (I, [P, L, I, I, P, P]),
    "sdc_symm_alloc": (I, [ctypes.c_ulonglong, ctypes.POINTER(ctypes.c_void_p)]),
    "sdc_symm_free": (I, [P]),
    "sdc_ipc_handle": (I, [P, P]),
    "sdc_ipc_handle_bytes": (I, []),
    "sdc_ipc_open": (I, [P, ctypes.POINTER(ctypes.c_void_p)]),
    "sdc_ipc_close": (I, [P]),
    "sdc_enable_peer_access": (I, [I]),
    "sdc_kv_page_checksums": (I, [P, L, L, I, P, I, ctypes.c_ulonglong, P, P]),
    "sdc_kv_pull_pages": (I, [P, L, P, L, L, I, P, P, I, ctypes.c_ulonglong, P, P, P, P, P]),
    "sdc_spot_check": (I, [P, L, P, P, L, P, I, I, P, I, P, I, F, F, P, P]),
    "sdc_gemm_bf16_grouped": (I, [P, L, P, P, I, I, I, I, P, L, P, P, P, P, P, P, I, U, U, U, U, F, F, F, F, F, P, I,
                                  I, I, U, P]),
    "sdc_silu_mul_bf16_bands": (I, [P, I, I, P, P, P, P]),
    "sdc_moe_plan": (I, [P, I, I, I, I, P, P, P, P, P, P, P]),
    "sdc_moe_gather": (I, [P, L, I, I, I, I, P, P, P, P, P, P]),
    "sdc_moe_combine": (I, [P, I, I, I, P, P, P, L, I, P]),
    "sdc_prep_rowblock": (I, [P, L, I, I, U, U, U, U, P, P, P, P, P]),
    "sdc_prep_colblock": (I, [P, L, I, I, U, U, U, U, P, P, P, P, P, P]),
    "sdc_transpose_bf16": (I, [P, L, I, I, P, P]),
    "sdc_dequant_weights": (I, [P, I, I, I, I, P, P, I, P, P]),
    "sdc_gemm_fp8_grouped": (I, [P, P, P, P, P, I, I, I, I, P, L, P, P, P, P, P, I, U, U, U, U, F, F, F, F, F, P, I,
                                 I, U, P]),
    "sdc_ep_receive_grouped": (I, [P, P, P, P, P, I, I, I, I, I, P, P, P, P, P, P, P, P, P]),
}


def _stale() -> bool:
    if not LIB_PATH.exists():
        return True
    if os.environ.get("SDCGUARD_NO_REBUILD") == "1":
        return False
    src = _PKG / "csrc"
    newest = max((p.stat().st_mtime for p in src.iterdir()), default=0.0)
    return LIB_PATH.stat().st_mtime < newest


def lib():
    """The loaded library, building it first if it is missing or older than its sources."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if _stale():
            from . import _build
            try:
                _build.build()
            except Exception as e:  # noqa: BLE001
                if not LIB_PATH.exists():
                    raise RuntimeError(f"sdcguard_b200 native library missing and could not be built: {e}") from e
        h = ctypes.CDLL(str(LIB_PATH))
        wrapped = _Lib(h)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(h, name, None)
            if fn is None:
                raise RuntimeError(f"{LIB_PATH.name} lacks {name}: rebuild with python -m sdcguard_b200._build")
            fn.restype = res
            fn.argtypes = args
            if not (name.endswith("_bytes") or name.endswith("_splits") or "_symm_" in name or "_ipc_" in name
                    or name.endswith("_peer_access") or "_capture" in name):
                setattr(wrapped, name, _Counted(fn))
        _lib = wrapped
        return _lib


WAIT_LIMIT_UNITS = ("attention", "ep_comm", "gemm_abft", "gemm_fp8", "tp_comm")
DEFAULT_WAIT_NS = 2_000_000_000


def set_wait_limit(ns: int = DEFAULT_WAIT_NS) -> None:
    """Deadline of every bounded device-side wait of this library's kernels (mbarrier phases, peer flags, band
    counters), in nanoseconds, on the CURRENT CUDA device. 2 s by default; a wait that runs out records an error
    code in the launch's error word and the kernel returns. Call outside stream capture (it is a synchronous copy
    to each compiled unit's own copy of the limit)."""
    h = lib()
    for unit in WAIT_LIMIT_UNITS:
        fn = getattr(h._h, f"sdc_set_wait_ns_{unit}")
        fn.restype = c_int
        fn.argtypes = [ctypes.c_ulonglong]
        check(fn(int(ns)), f"sdc_set_wait_ns_{unit}")


def available() -> bool:
    try:
        lib()
        return True
    except Exception:  # noqa: BLE001
        return False


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what} failed with code {rc}")
