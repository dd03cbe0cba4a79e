"""Bit fingerprints of tensors (two 64-bit sums per tensor; `csrc/fingerprint.cu`).

    fp = fingerprint([w1, w2, ...])        # (n, 2) int64 on the tensors' device, no host synchronisation
    fingerprint_host(t)                    # the same two numbers computed with NumPy (CPU tensors, tests)

F0 = sum of the 8-byte words mod 2^64 (a single flipped bit always changes it); F1 = sum of fmix64(word XOR key(i))
mod 2^64 with a position key (swaps and paired errors change it). CUDA tensors go through the kernel; CPU tensors
(gloo ranks, CPU models) through the NumPy restatement of the same formula.
"""
from __future__ import annotations

from typing import Sequence

import numpy as np
import torch

from .. import _native

GOLDEN = 0x9E3779B97F4A7C15
MASK = (1 << 64) - 1


def _fmix64(k: np.ndarray) -> np.ndarray:
    k = k.copy()
    k ^= k >> np.uint64(33)
    k *= np.uint64(0xff51afd7ed558ccd)
    k ^= k >> np.uint64(33)
    k *= np.uint64(0xc4ceb9fe1a85ec53)
    k ^= k >> np.uint64(33)
    return k


def _words(t: torch.Tensor) -> np.ndarray:
    b = t.detach().contiguous().cpu().view(torch.uint8).numpy().reshape(-1)
    pad = (-b.size) % 8
    if pad:
        b = np.concatenate([b, np.zeros(pad, np.uint8)])
    return b.view(np.uint64)


def fingerprint_host(t: torch.Tensor, seed: int = 0) -> tuple[int, int]:
    w = _words(t)
    with np.errstate(over="ignore"):
        idx = np.arange(1, w.size + 1, dtype=np.uint64)
        keys = idx * np.uint64(GOLDEN) + np.uint64(seed & MASK)
        f0 = int(np.sum(w, dtype=np.uint64))
        f1 = int(np.sum(_fmix64(w ^ keys), dtype=np.uint64))
    return f0, f1


def _signed(v: int) -> int:
    return v - (1 << 64) if v >= (1 << 63) else v


def fingerprint(tensors: Sequence[torch.Tensor], seed: int = 0) -> torch.Tensor:
    """(n, 2) int64 fingerprints (bit patterns of the u64 sums) of the tensors, on their device."""
    tensors = list(tensors)
    if not tensors:
        return torch.zeros(0, 2, dtype=torch.int64)
    dev = tensors[0].device
    if dev.type != "cuda":
        return torch.tensor([[_signed(v) for v in fingerprint_host(t, seed)] for t in tensors], dtype=torch.int64)
    items = torch.empty(len(tensors), 2, dtype=torch.int64, pin_memory=True)
    mx = 1
    for i, t in enumerate(tensors):
        if t.device != dev or not t.is_contiguous():
            raise ValueError("fingerprint: tensors must be contiguous and on one device")
        nbytes = t.numel() * t.element_size()
        items[i, 0] = t.data_ptr()
        items[i, 1] = nbytes
        mx = max(mx, nbytes)
    items_dev = items.to(dev, non_blocking=True)
    out = torch.empty(len(tensors), 2, dtype=torch.int64, device=dev)
    _native.check(_native.lib().sdc_fingerprint_many(items_dev.data_ptr(), len(tensors), mx, seed & MASK,
                                                      out.data_ptr(), torch.cuda.current_stream(dev).cuda_stream),
                  "fingerprint")
    out._keepalive = (items, items_dev)          # the copies must finish before the buffers are reused
    return out
