"""Math-mode screen: one matmul per arithmetic mode (bf16, fp16, tf32, fp32, fp64, int8, fp8), each checked against a
float64 CPU reference of the same inputs, with a noise model of that mode's accumulation.

    python -m sdcguard_b200.tools.modes                  # every mode on cuda:0, the six input variants
    python -m sdcguard_b200.tools.modes --modes fp32 fp64 --json

A GPU can be wrong in one mode and right in the others (different units: CUDA-core FMA for fp32 / fp64, tensor cores
for the rest, integer tensor cores for int8). Inputs are exactly representable in the mode (bf16 / fp16 / fp8 values,
TF32-exact fp32 values, small integers), so the only error left is the accumulation's own rounding, and results are
kept wide (fp32, fp64, int32). For every row and 128-column block the plain and the +-1-signed sums of the result are
compared with the reference's; the noise of a block sum is

    u (|a_row| . |B|_block + sqrt(k) |C|_block)          (IEEE FMA accumulation, u = 2^-24 or 2^-53)
  + u (k / n_step) |C|_block                              (tensor cores: n_step products added per step and the sum
                                                           truncated toward zero; Blackwell: 16 per step in bf16 /
                                                           fp16, 8 in tf32, 32 in fp8, keeping fp32-level bits)

and a block is wrong above 6 units. int8 must match exactly. Six input variants (normal, uniform, sparse, laplace at
several scales, all zero-mean, because truncation errors of same-signed inputs add up).

Reference: src/sdcguard/modes.py:1-34 (the mode list, the truncation model from Khattak and Mikaitis, and the
6-unit alarm), `screen` :383.
"""
from __future__ import annotations

import argparse
import json
import math
import time
from typing import Optional

import torch

from ..numerics import abft

ALARM = 6.0
MODES = ("bf16", "fp16", "tf32", "fp32", "fp64", "int8", "fp8")
VARIANTS = (("normal", 1.0), ("uniform", 2.0 ** -8), ("sparse", 2.0 ** 6), ("normal", 2.0 ** 8),
            ("laplace", 2.0 ** -4), ("uniform", 1.0))
SHAPE = {"cuda": (2048, 1024, 2048), "cpu": (256, 256, 256)}      # (m, k, n)
FP8_K = 256
STEP = {"bf16": 16, "fp16": 16, "tf32": 8, "fp8": 32}                # products per truncation step (sm_100)


def _sample(shape, dist: str, scale: float, g: torch.Generator) -> torch.Tensor:
    if dist == "normal":
        x = torch.randn(shape, generator=g)
    elif dist == "uniform":
        x = torch.rand(shape, generator=g) * 2 - 1
    elif dist == "sparse":
        x = torch.randn(shape, generator=g) * (torch.rand(shape, generator=g) < 0.1)
    elif dist == "laplace":
        u = torch.rand(shape, generator=g).clamp(1e-7, 1 - 1e-7) - 0.5
        x = (-torch.sign(u) * torch.log1p(-2 * u.abs())).clamp(-20, 20)
    else:
        raise ValueError(dist)
    return x * scale


def _exact(mode: str, x: torch.Tensor) -> torch.Tensor:
    """Inputs representable in the mode, as float64 values."""
    if mode == "bf16":
        return x.to(torch.bfloat16).double()
    if mode == "fp16":
        return x.clamp(-6e4, 6e4).to(torch.float16).double()
    if mode == "tf32":
        return (x.float().view(torch.int32) & -8192).view(torch.float32).double()
    if mode == "fp32":
        return x.float().double()
    if mode == "fp8":
        y = x / (x.abs().max() / 240 + 1e-30)                       # into E4M3's range, away from subnormals
        y = torch.where(y.abs() < 2.0 ** -6, torch.zeros_like(y), y)
        return y.to(torch.float8_e4m3fn).double()
    if mode == "int8":
        return (x / (x.abs().max() + 1e-30) * 127).round().clamp(-127, 127).double()
    return x.double()


def device_matmul(mode: str, a: torch.Tensor, b: torch.Tensor, device) -> torch.Tensor:
    """The mode's GEMM on the device: a (m, k), b (k, n) float64 holding exact values; result in fp32 / fp64 /
    int32."""
    if mode == "int8":
        return torch._int_mm(a.to(device, torch.int8), b.to(device, torch.int8))
    if mode == "fp8":
        f8 = torch.float8_e4m3fn
        one = torch.ones((), device=device)
        bb = b.t().contiguous().to(device, f8).t()
        return torch._scaled_mm(a.to(device, f8), bb, scale_a=one, scale_b=one, out_dtype=torch.float32)
    dt = {"bf16": torch.bfloat16, "fp16": torch.float16, "tf32": torch.float32, "fp32": torch.float32,
          "fp64": torch.float64}[mode]
    prev = torch.backends.cuda.matmul.allow_tf32
    try:
        torch.backends.cuda.matmul.allow_tf32 = mode == "tf32"
        if mode in ("bf16", "fp16"):       # fp32 result: out_dtype keeps the accumulator's bits
            if torch.device(device).type != "cuda":     # CPU: the exact values in an fp32 matmul
                return torch.mm(a.to(device, dt).float(), b.to(device, dt).float())
            return torch.mm(a.to(device, dt), b.to(device, dt), out_dtype=torch.float32)
        return a.to(device, dt) @ b.to(device, dt)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def judge(mode: str, a: torch.Tensor, b: torch.Tensor, c: torch.Tensor, on_gpu: bool) -> dict:
    """Block-sum scores of result c (any dtype) against the float64 product of a and b."""
    ref = a @ b
    cd = c.double().cpu()
    m, n = ref.shape
    nb = -(-n // 128)
    pad = nb * 128 - n
    sgn = abft.sign_vector(abft.sign_mask(), dtype=torch.float64, device="cpu")

    def blocks(x):
        return torch.nn.functional.pad(x, (0, pad)).view(m, nb, 128)

    if mode == "int8":
        wrong = int((cd != ref).sum())
        return {"z": math.inf if wrong else 0.0, "wrong_blocks": wrong, "checks": m * n}
    R, C = blocks(ref), blocks(cd)
    dp = (C.sum(-1) - R.sum(-1)).abs()
    ds = ((C - R) * sgn).sum(-1).abs()
    k = a.shape[1]
    u = 2.0 ** -53 if mode == "fp64" else 2.0 ** -24
    babs = torch.nn.functional.pad(b.abs(), (0, pad)).view(k, nb, 128).sum(-1)        # (k, nb)
    cn = C.abs().sum(-1)
    noise = u * (a.abs() @ babs + math.sqrt(k) * torch.linalg.vector_norm(C, dim=-1))
    if on_gpu and mode in STEP:
        noise = noise + u * (k / STEP[mode]) * cn
    noise = noise + 1e-300
    z = torch.maximum(dp, ds) / noise
    nonfinite = ~torch.isfinite(C).all(-1)
    z = torch.where(nonfinite, torch.full_like(z, math.inf), z)
    return {"z": float(z.max()), "wrong_blocks": int((z > ALARM).sum()), "checks": int(z.numel())}


def check_once(mode: str, device, variant: tuple, seed: int, shape: Optional[tuple] = None) -> dict:
    dev = torch.device(device)
    m, k, n = shape or SHAPE["cuda" if dev.type == "cuda" else "cpu"]
    if mode == "fp8":
        k = min(k, FP8_K)
    g = torch.Generator().manual_seed(seed)
    a = _exact(mode, _sample((m, k), *variant, g))
    b = _exact(mode, _sample((k, n), *variant, g))
    t0 = time.perf_counter()
    c = device_matmul(mode, a, b, dev)
    if dev.type == "cuda":
        torch.cuda.synchronize(dev)
    r = judge(mode, a, b, c, dev.type == "cuda")
    r.update(mode=mode, variant=f"{variant[0]}x{variant[1]:g}", seed=seed, shape=(m, k, n),
             ms=round((time.perf_counter() - t0) * 1e3, 2))
    return r


def supported(mode: str, device) -> Optional[str]:
    dev = torch.device(device)
    if dev.type != "cuda":
        return None if mode in ("fp32", "fp64", "bf16") else "needs a GPU"
    if mode == "fp8" and not hasattr(torch, "_scaled_mm"):
        return "torch._scaled_mm missing"
    if mode == "int8" and not hasattr(torch, "_int_mm"):
        return "torch._int_mm missing"
    return None


def screen(device="cuda:0", modes=MODES, variants=VARIANTS, seed: int = 0, shape: Optional[tuple] = None) -> dict:
    """Every mode over every variant: per mode the worst score, wrong blocks, checks, and the failing cases with
    what it takes to replay them (mode, variant, seed, shape)."""
    out = {"device": str(device), "modes": {}, "skipped": {}}
    for mode in modes:
        why = supported(mode, device)
        if why:
            out["skipped"][mode] = why
            continue
        rows = []
        for i, v in enumerate(variants):
            try:
                rows.append(check_once(mode, device, v, seed * 100 + i, shape))
            except RuntimeError as e:
                out["skipped"][mode] = f"unsupported here: {str(e).splitlines()[0][:200]}"
                rows = []
                break
        if not rows:
            continue
        bad = [r for r in rows if r["wrong_blocks"]]
        out["modes"][mode] = {"worst_z": max(r["z"] for r in rows), "wrong_blocks": sum(r["wrong_blocks"] for r in rows),
                              "checks": sum(r["checks"] for r in rows), "verdict": "FAIL" if bad else "pass",
                              "failing": [{k: r[k] for k in ("variant", "seed", "shape", "z")} for r in bad]}
    out["verdict"] = "FAIL" if any(m["verdict"] == "FAIL" for m in out["modes"].values()) else "pass"
    return out


def replay(case: dict, mode: str, device="cuda:0") -> dict:
    """Rerun one failing case of a report (its variant name, seed and shape)."""
    dist, scale = case["variant"].split("x")
    return check_once(mode, device, (dist, float(scale)), case["seed"], tuple(case["shape"]))


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m sdcguard_b200.tools.modes")
    ap.add_argument("--device", default="cuda:0" if torch.cuda.is_available() else "cpu")
    ap.add_argument("--modes", nargs="*", default=list(MODES))
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--json", action="store_true")
    a = ap.parse_args(argv)
    r = screen(a.device, a.modes, seed=a.seed)
    if a.json:
        print(json.dumps(r))
    else:
        for mode, d in r["modes"].items():
            print(f"{mode:5s} {d['verdict']:4s} worst z {d['worst_z']:.3g}  checks {d['checks']}")
        for mode, why in r["skipped"].items():
            print(f"{mode:5s} skipped: {why}")
    return 0 if r["verdict"] == "pass" else 1


if __name__ == "__main__":
    raise SystemExit(main())
