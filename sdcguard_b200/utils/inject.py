"""Seeded host-side fault injection: corrupts outputs of matrix multiplications (or any tensor) the way hardware
faults corrupt them, so that the detectors can be measured. Nothing here touches a GPU in a way that can fault it:
the injector changes values of ordinary tensors after the operation that produced them.

Fault models (`FaultModel`):
  * "bitflip": one bit of one element.
  * "nvidia": the output-corruption mix published by NVIDIA for GPU faults, as the reference uses it
    (src/sdcguard/inject.py:54-92): a value becomes zero (50.68%), has a bit flipped (48.31%) or becomes NaN/Inf
    (1.01%); the corrupted elements form a chunk of 32 consecutive values (a warp) with a period of 1-16, or a
    128 x 128 tile.

`FaultInjector` is a TorchDispatchMode that corrupts the result of aten mm / addmm / bmm / baddbmm / linear calls
with a given probability per call and records every injection (op index, position, kind, bit, old and new value).
`flip_bit_` is the primitive used by the serving campaign and the KV / all-to-all payload injections.

Reference: `FaultModel` :54, `fault_model` :72, `corrupt_` :161, `FaultInjector` :198 (src/sdcguard/inject.py).
"""
from __future__ import annotations

import random
from dataclasses import dataclass
from typing import Optional

import torch
from torch.utils._python_dispatch import TorchDispatchMode

NVIDIA_MIX = (("zero", 0.5068), ("bitflip", 0.4831), ("nonfinite", 0.0101))
_INT_VIEW = {torch.float32: torch.int32, torch.float16: torch.int16, torch.bfloat16: torch.int16,
             torch.float64: torch.int64}


def flip_bit_(t: torch.Tensor, flat_index: int, bit: int) -> tuple[float, float]:
    """Flips `bit` of element `flat_index` of floating tensor t in place; returns (old, new) values."""
    iv = _INT_VIEW[t.dtype]
    nbits = torch.iinfo(iv).bits
    flat = t.view(-1)
    old = float(flat[flat_index])
    w = flat.view(iv)
    mask = (1 << bit) if bit < nbits - 1 else -(1 << (nbits - 1))
    w[flat_index] ^= mask
    return old, float(flat[flat_index])


@dataclass
class FaultModel:
    kind: str = "bitflip"                      # "bitflip" or "nvidia"
    tile_fraction: float = 0.1                 # "nvidia": share of events that hit a 128x128 tile

    def sample(self, rng: random.Random) -> str:
        if self.kind == "bitflip":
            return "bitflip"
        r, acc = rng.random(), 0.0
        for k, p in NVIDIA_MIX:
            acc += p
            if r < acc:
                return k
        return NVIDIA_MIX[-1][0]


def corrupt_(t: torch.Tensor, rng: random.Random, model: FaultModel) -> dict:
    """Corrupts t in place according to the model; returns a description of the injection."""
    n = t.numel()
    nbits = torch.iinfo(_INT_VIEW[t.dtype]).bits
    kind = model.sample(rng)
    if model.kind == "bitflip":
        i, b = rng.randrange(n), rng.randrange(nbits)
        old, new = flip_bit_(t, i, b)
        return {"kind": "bitflip", "index": i, "bit": b, "old": old, "new": new, "elements": [i]}
    flat = t.view(-1)
    if rng.random() < model.tile_fraction and t.dim() >= 2 and t.shape[-1] >= 128 and t.numel() // t.shape[-1] >= 128:
        cols = t.shape[-1]
        rows = n // cols
        r0, c0 = rng.randrange(0, rows - 127), rng.randrange(0, cols - 127)
        elems = [(r0 + r) * cols + c0 + c for r in range(128) for c in range(128)]
        shape = "tile128"
    else:
        period = rng.randint(1, 16)
        start = rng.randrange(n)
        elems = [start + j * period for j in range(32) if start + j * period < n]
        shape = f"warp32/p{period}"
    bit = rng.randrange(nbits)
    for i in elems:
        if kind == "zero":
            flat[i] = 0
        elif kind == "nonfinite":
            flat[i] = float("nan") if rng.random() < 0.5 else float("inf")
        else:
            flip_bit_(t, i, bit)
    return {"kind": kind, "shape": shape, "elements": elems[:8], "count": len(elems), "bit": bit}


_MM_OPS = None


def _mm_ops():
    global _MM_OPS
    if _MM_OPS is None:
        a = torch.ops.aten
        _MM_OPS = {a.mm.default, a.addmm.default, a.bmm.default, a.baddbmm.default}
    return _MM_OPS


class FaultInjector(TorchDispatchMode):
    """Corrupts matmul results with probability `rate` per call (seeded). `injections` lists what was done."""

    def __init__(self, rate: float = 0.01, seed: int = 0, model: Optional[FaultModel] = None):
        super().__init__()
        self.rate = rate
        self.rng = random.Random(seed)
        self.model = model or FaultModel()
        self.calls = 0
        self.injections: list[dict] = []
        self.enabled = True

    def __torch_dispatch__(self, func, types, args=(), kwargs=None):
        out = func(*args, **(kwargs or {}))
        if func in _mm_ops() and isinstance(out, torch.Tensor) and out.dtype in _INT_VIEW:
            idx = self.calls
            self.calls += 1
            if self.enabled and self.rng.random() < self.rate:
                d = corrupt_(out, self.rng, self.model)
                d["call"] = idx
                self.injections.append(d)
        return out
