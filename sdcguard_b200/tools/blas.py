"""Every cuBLASLt algorithm a linear layer's matmul could run, each checked against float64, and the cuBLAS calls
GPU burn-in tools make.

    from sdcguard_b200.tools.blas import sweep, legacy
    r = sweep(4096, 4096, 2048)          # out features, in features, tokens
    r["wrong_algorithms"]                # [] when every algorithm wrote every element and computed correctly
    python -m sdcguard_b200.tools.blas --m 4096 --k 4096 --n 2048 --dtype bf16
    python -m sdcguard_b200.tools.blas --legacy 2048

The library picks one algorithm per shape, type and setting; a defect in another algorithm shows up only when the
heuristic switches to it, so a one-GEMM burn-in never sees it. `sweep` runs every algorithm the heuristic offers (up
to 16, plus the first again with a 1x1x1 cluster) through the native host probe (`csrc/host/blas_probe.cpp`, linked to
cuBLASLt), each into an output pre-filled with NaN: every element must have been written, and sampled rows must be
within a rigorous bound of the float64 product (fp32 accumulation: u (sqrt(k) + 2) |a| . |b| plus the output
rounding). `legacy` runs Hgemm / Sgemm / Sgemm (tensor-op) / Dgemm / GemmEx fp16 / GemmEx bf16 on DCGM-style inputs
and compares sampled columns with float64; `fresh_memory_nonzero` says whether a fresh allocation is zeroed.

Reference: src/sdcguard/blas.py:1-22 (`sweep` :152), experiments/h2h_probe.cpp:1-30.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math

import torch

_HOST = None
DT = {"fp16": (0, torch.float16, 2.0 ** -11), "bf16": (1, torch.bfloat16, 2.0 ** -8), "fp32": (2, torch.float32,
                                                                                               2.0 ** -24)}
LEGACY = {"hgemm": (0, torch.float16), "sgemm": (1, torch.float32), "sgemm_tc": (2, torch.float32),
          "dgemm": (3, torch.float64), "gemmex_fp16": (4, torch.float16), "gemmex_bf16": (5, torch.bfloat16)}
MAX_ALGOS = 16
SAMPLE_ROWS = 64


def host():
    """The host probe library (built by `sdcguard_b200._build`); torch is imported first so the CUDA libraries it
    loaded satisfy the probe's."""
    global _HOST
    if _HOST is None:
        from .. import _build
        path = _build.HOST_LIB
        if not path.exists():
            _build.build_host()
        lib = ctypes.CDLL(str(path))
        P, I, L = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong
        lib.sdc_blaslt_sweep.restype = I
        lib.sdc_blaslt_sweep.argtypes = [I, I, I, I, P, P, P, P, L, I, P, I, P]
        lib.sdc_blas_legacy.restype = I
        lib.sdc_blas_legacy.argtypes = [I, I, P, P, P, P]
        lib.sdc_fresh_nonzero.restype = L
        lib.sdc_fresh_nonzero.argtypes = [L]
        _HOST = lib
    return _HOST


def bound(a: torch.Tensor, b: torch.Tensor, ref: torch.Tensor, u_out: float) -> torch.Tensor:
    """Rigorous error bound of k fp32-accumulated products in any summation order and grouping (k u |a| . |b|, with
    a 1% margin for the second-order term), plus one output rounding."""
    k = a.shape[-1]
    mag = a.abs() @ b.abs().t()
    return 1.01 * k * 2.0 ** -24 * mag + u_out * ref.abs() + 1e-30


def sweep(m: int, k: int, n: int, dtype: str = "bf16", device: str = "cuda:0", seed: int = 0,
          force_1x1: bool = True, ws_mb: int = 64) -> dict:
    """y (n, m) = x (n, k) @ W (m, k)^T with every offered algorithm. Returns per-algorithm results and the list of
    wrong ones (unwritten elements, or sampled rows outside the bound)."""
    code, tdt, u_out = DT[dtype]
    dev = torch.device(device)
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(m, k, generator=g).to(tdt)
    x = torch.randn(n, k, generator=g).to(tdt)
    wd, xd = w.to(dev), x.to(dev)
    out = torch.empty(MAX_ALGOS + 1, n, m, dtype=tdt, device=dev)
    ws = torch.empty(ws_mb << 20, dtype=torch.uint8, device=dev)
    info = (ctypes.c_int * (8 * (MAX_ALGOS + 1)))()
    st = torch.cuda.current_stream(dev).cuda_stream
    offered = host().sdc_blaslt_sweep(m, k, n, code, wd.data_ptr(), xd.data_ptr(), out.data_ptr(), ws.data_ptr(),
                                      ws.numel(), MAX_ALGOS, info, int(force_1x1), st)
    torch.cuda.synchronize(dev)
    if offered < 0:
        return {"error": f"probe returned {offered}", "shape": (m, k, n), "dtype": dtype}
    runs = offered + (1 if force_1x1 and offered else 0)
    rows = torch.randperm(n, generator=g)[:SAMPLE_ROWS]
    ref = x.double()[rows] @ w.double().t()
    bnd = bound(x.double()[rows], w.double(), ref, u_out)
    algos, wrong = [], []
    for i in range(runs):
        r = list(info[8 * i: 8 * i + 8])
        y = out[i]
        unwritten = int(torch.isnan(y).sum()) if r[0] == 0 else None
        d = {"run": i, "status": r[0], "algo_id": r[1], "tile_id": r[2], "splitk": r[3], "stages_id": r[4],
             "cluster_shape_id": r[5], "reduction_scheme": r[6], "workspace_kib": r[7],
             "forced_1x1": i == offered}
        if r[0] == 0:
            z = ((y[rows.to(dev)].double().cpu() - ref).abs() / bnd)
            d.update(unwritten=unwritten, worst_score=float(z.nan_to_num(math.inf).max()),
                     wrong_samples=int((z > 1).sum() + torch.isnan(z).sum()))
            if unwritten or d["wrong_samples"]:
                wrong.append(i)
        algos.append(d)
    return {"shape": {"out_features": m, "in_features": k, "tokens": n}, "dtype": dtype, "offered": offered,
            "algorithms": algos, "wrong_algorithms": wrong, "verdict": "FAIL" if wrong else "pass"}


def legacy(n: int = 2048, device: str = "cuda:0", kinds=tuple(LEGACY), seed: int = 10) -> dict:
    """The burn-in tools' cuBLAS calls on square n, inputs in [0, 10) like theirs; sampled columns vs float64."""
    dev = torch.device(device)
    g = torch.Generator().manual_seed(seed)
    a64 = torch.randint(0, 1000000, (n, n), generator=g).double() / 100000.0
    b64 = torch.randint(0, 1000000, (n, n), generator=g).double() / 100000.0
    cols = torch.randperm(n, generator=g)[:16]
    out = {}
    st = torch.cuda.current_stream(dev).cuda_stream
    for name in kinds:
        code, dt = LEGACY[name]
        # column-major operands: pass the transposes' storage (row-major A^T is column-major A)
        a, b = a64.to(dt), b64.to(dt)
        ad, bd = a.t().contiguous().to(dev), b.t().contiguous().to(dev)
        c = torch.full((n, n), float("nan"), dtype=dt, device=dev)
        s = host().sdc_blas_legacy(code, n, ad.data_ptr(), bd.data_ptr(), c.data_ptr(), st)
        torch.cuda.synchronize(dev)
        if s != 0:
            out[name] = {"status": s}
            continue
        got = c.t().double().cpu()[:, cols]               # C column-major -> row-major view
        ref = a.double() @ b.double()[:, cols]
        tol = 5e-2 * (1 + ref.abs()) if dt in (torch.float16, torch.bfloat16) else 1e-4 * (1 + ref.abs())
        bad = int(((got - ref).abs() > tol).sum() + torch.isnan(got).sum())
        out[name] = {"status": 0, "unwritten": int(torch.isnan(c).sum()), "wrong_sampled": bad,
                     "verdict": "FAIL" if bad else "pass"}
    return out


def fresh_memory_nonzero(nbytes: int = 64 << 20) -> int:
    return int(host().sdc_fresh_nonzero(nbytes))


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m sdcguard_b200.tools.blas")
    ap.add_argument("--m", type=int, default=4096)
    ap.add_argument("--k", type=int, default=4096)
    ap.add_argument("--n", type=int, default=2048)
    ap.add_argument("--dtype", default="bf16", choices=list(DT))
    ap.add_argument("--device", default="cuda:0")
    ap.add_argument("--legacy", type=int, default=0, help="also run the burn-in calls on this square size")
    a = ap.parse_args(argv)
    r = {"sweep": sweep(a.m, a.k, a.n, a.dtype, a.device)}
    if a.legacy:
        r["legacy"] = legacy(a.legacy, a.device)
        r["fresh_memory_nonzero_bytes"] = fresh_memory_nonzero()
    print(json.dumps(r))
    bad = r["sweep"].get("wrong_algorithms") or any(v.get("verdict") == "FAIL" for v in r.get("legacy", {}).values())
    return 1 if bad else 0


if __name__ == "__main__":
    raise SystemExit(main())
