"""Calibration of the fp32-accumulator noise model of the checked GEMM on this GPU.

    python -m sdcguard_b200.tools.calibrate [--out calib.json] [--reps 3]

Runs clean checked GEMMs over a grid of shapes (decode- and prefill-sized M, the N and K of the served and trained
models, split-K and CTA-pair paths included) and input distributions (normal, uniform, heavy-tailed, wide dynamic
range, near-cancelling rows, with and without bias), with the coefficients scaled by `--scale`, and records the
worst score per case. The score is linear in the coefficients (z = |expected - actual| / den, den proportional to
them apart from the 1e-20 floor), so the worst clean score at scale 1 says how far the coefficients can come down:
`suggested_scale` puts the worst calibration score at `--target` (default 0.5, twelve times below the alarm line
of 6). The held-out evidence that a chosen scale raises no false alarm is separate: the clean serving run of the
bench and the campaign's clean checks, which this tool never sees.

Reference: the reference calibrates its precise mode on held-out runs before freezing it
(experiments/calibrate.py, docs/METHOD.md:309-312, :380-398); here the same discipline picks C1 and C2.
"""
from __future__ import annotations

import argparse
import json
import math

import torch

from ..numerics import abft
from ..ops import gemm

SHAPES = [  # (M, N, K): decode and prefill sizes of Qwen3-0.6B, Llama-3-8B shards, GPT-2 training shapes
    (64, 4096, 1024), (256, 4096, 1024), (256, 1024, 2048), (256, 6144, 1024), (256, 1024, 3072),
    (64, 4096, 14336), (512, 3072, 768), (2048, 768, 3072), (4096, 4096, 1024), (4096, 6144, 4096),
    (8192, 1024, 3072), (16384, 768, 768), (1024, 28672, 4096),
]
DISTRIBUTIONS = ("normal", "uniform", "heavy", "wide", "cancel", "softmax_grad")
# training GEMMs with a long K (the token count): dW of the projections and of a 50304-word LM head at 32 x 512
# tokens, and dX of that head (K = the vocabulary)
TRAIN_SHAPES = [(2304, 768, 16384), (768, 3072, 16384), (3072, 768, 16384), (50304, 768, 16384),
                (16384, 768, 50304), (16384, 2304, 768)]


def _inputs(kind: str, m: int, n: int, k: int, g: torch.Generator, dev) -> tuple[torch.Tensor, torch.Tensor]:
    if kind == "normal":
        x, w = torch.randn(m, k, generator=g, device=dev), torch.randn(n, k, generator=g, device=dev) * 0.02
    elif kind == "uniform":
        x = torch.rand(m, k, generator=g, device=dev) * 2 - 1
        w = (torch.rand(n, k, generator=g, device=dev) * 2 - 1) * 0.05
    elif kind == "heavy":          # Student-t-like tails: a few very large activations per row
        x = torch.randn(m, k, generator=g, device=dev) / (torch.rand(m, k, generator=g, device=dev) + 0.05)
        w = torch.randn(n, k, generator=g, device=dev) * 0.02
    elif kind == "wide":           # rows and columns over many binades
        ex = torch.randint(-12, 12, (m, 1), generator=g, device=dev).float()
        ew = torch.randint(-6, 6, (n, 1), generator=g, device=dev).float()
        x = torch.randn(m, k, generator=g, device=dev) * torch.exp2(ex)
        w = torch.randn(n, k, generator=g, device=dev) * 0.02 * torch.exp2(ew)
    elif kind == "softmax_grad":   # rows of a softmax cross-entropy gradient: tiny, one-signed, a few large negatives
        x = torch.rand(m, k, generator=g, device=dev) * 2e-9
        hit = torch.rand(m, k, generator=g, device=dev) < 2e-4
        x[hit] = -6e-5
        w = torch.randn(n, k, generator=g, device=dev)
    else:                          # rows whose dot products nearly cancel
        x = torch.randn(m, k, generator=g, device=dev)
        x[:, k // 2:] = -x[:, : k - k // 2].flip(1)
        w = torch.randn(n, k, generator=g, device=dev) * 0.02
        w[:, k // 2:] = w[:, : k - k // 2].flip(1)
    return x.to(dev).bfloat16(), w.to(dev).bfloat16()


def run(device="cuda", reps: int = 2, scale: float = 1.0, target: float = 0.5, shapes=None) -> dict:
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(20261202)
    rows, worst = [], 0.0
    checks = 0
    for (m, n, k) in shapes or SHAPES:
        for kind in DISTRIBUTIONS:
            for bias in (False, True):
                x, w = _inputs(kind, m, n, k, g, dev)
                b = (torch.randn(n, generator=g, device=dev) * 0.1).bfloat16() if bias else None
                cw = gemm.CheckedWeight(w, b, c1=abft.C1 * scale, c2=abft.C2 * scale, c3=abft.C3 * scale)
                table = gemm.StateTable(dev, 1)
                slot = table.add("calibration", cw.nb)
                for _ in range(reps):
                    gemm.checked_linear(x, cw, table.state, slot)
                r = table.read(reset=True)[0]
                z = r["z"] if math.isfinite(r["z"]) else float("inf")
                checks += reps * m * cw.nb * 2
                worst = max(worst, z)
                rows.append({"m": m, "n": n, "k": k, "inputs": kind, "bias": bias, "worst_z": round(z, 5),
                             "unjudged": r["unjudged"]})
                del x, w, cw
        torch.cuda.empty_cache()
    return {"gpu": torch.cuda.get_device_name(dev), "coefficients": {"c1": abft.C1, "c2": abft.C2, "c3": abft.C3},
            "scale": scale, "checks": checks, "worst_z": round(worst, 5),
            "suggested_scale": round(scale * worst / target, 4) if worst > 0 else None, "target": target,
            "cases": rows}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m sdcguard_b200.tools.calibrate")
    ap.add_argument("--device", default="cuda")
    ap.add_argument("--reps", type=int, default=2)
    ap.add_argument("--scale", type=float, default=1.0, help="multiplier on the coefficients C1, C2, C3")
    ap.add_argument("--target", type=float, default=0.5)
    ap.add_argument("--out")
    ap.add_argument("--set", choices=("serve", "train", "all"), default="serve",
                    help="shape grid: serving and prefill shapes, long-K training shapes, or both")
    a = ap.parse_args(argv)
    shapes = {"serve": SHAPES, "train": TRAIN_SHAPES, "all": SHAPES + TRAIN_SHAPES}[a.set]
    res = run(a.device, a.reps, a.scale, a.target, shapes=shapes)
    text = json.dumps(res, indent=1)
    if a.out:
        with open(a.out, "w") as f:
            f.write(text)
    print(json.dumps({k: v for k, v in res.items() if k != "cases"}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
