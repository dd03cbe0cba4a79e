"""Checksummed KV-page transfer (`csrc/kv_transfer.cu`): per-page 64-bit checksums of local pages and a peer-memory
pull that hashes pages as they arrive and compares them with the producer's checksums.

`page_checksum_reference` is the same function in plain PyTorch/NumPy (tests and CPU tooling).
"""
from __future__ import annotations

from typing import Optional

import numpy as np
import torch

from .. import _native

DEFAULT_SEED = 0x5DC9_0A2D_B200_0001


def _s(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _geometry(cache: torch.Tensor):
    """cache: (layers, blocks, ...) bf16 -> (layers, layer stride bytes, page bytes)."""
    L = cache.shape[0]
    page_bytes = cache[0, 0].numel() * cache.element_size()
    return L, cache.stride(0) * cache.element_size(), page_bytes


def page_checksums(cache: torch.Tensor, pages: torch.Tensor, seed: int = DEFAULT_SEED,
                   out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """(n,) int64 (bit pattern of uint64) checksums of cache pages `pages` (int32 on the device)."""
    L, ls, pb = _geometry(cache)
    n = pages.numel()
    if out is None:
        out = torch.empty(n, dtype=torch.int64, device=cache.device)
    _native.check(_native.lib().sdc_kv_page_checksums(cache.data_ptr(), ls, pb, L, pages.data_ptr(), n,
                                                      seed & 0xFFFFFFFFFFFFFFFF, out.data_ptr(), _s(cache)),
                  "kv page checksums")
    return out


def pull_pages(src_cache: torch.Tensor, dst_cache: torch.Tensor, src_pages: torch.Tensor, dst_pages: torch.Tensor,
               want: torch.Tensor, seed: int = DEFAULT_SEED, state_row: Optional[torch.Tensor] = None,
               acc: Optional[torch.Tensor] = None):
    """Copy pages from src_cache (may be another GPU's memory mapped into this process) into dst_cache, hash them
    on arrival and compare with `want`. Returns (received checksums, per-page result: 1 match / 2 mismatch)."""
    L, sls, pb = _geometry(src_cache)
    L2, dls, pb2 = _geometry(dst_cache)
    if L != L2 or pb != pb2:
        raise ValueError("source and destination caches have different page geometry")
    n = src_pages.numel()
    if acc is None:
        acc = torch.empty(n, dtype=torch.int64, device=dst_cache.device)
    res = torch.empty(n, dtype=torch.int32, device=dst_cache.device)
    _native.check(_native.lib().sdc_kv_pull_pages(
        src_cache.data_ptr(), sls, dst_cache.data_ptr(), dls, pb, L, src_pages.data_ptr(), dst_pages.data_ptr(), n,
        seed & 0xFFFFFFFFFFFFFFFF, want.data_ptr(), acc.data_ptr(), res.data_ptr(),
        None if state_row is None else state_row.data_ptr(), _s(dst_cache)), "kv pull pages")
    return acc, res


_M = np.uint64(0xFFFFFFFFFFFFFFFF)


def _fmix64(k: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        k = k ^ (k >> np.uint64(33))
        k = k * np.uint64(0xFF51AFD7ED558CCD)
        k = k ^ (k >> np.uint64(33))
        k = k * np.uint64(0xC4CEB9FE1A85EC53)
        k = k ^ (k >> np.uint64(33))
    return k


def page_checksum_reference(cache: torch.Tensor, page: int, seed: int = DEFAULT_SEED) -> int:
    """The page checksum in NumPy: sum over the page's 8-byte words (numbered across layers) of
    fmix64(word ^ ((w + 1) * golden + seed)) mod 2^64."""
    words = [cache[l, page].contiguous().view(torch.int64).flatten().cpu().numpy().view(np.uint64)
             for l in range(cache.shape[0])]
    w = np.concatenate(words)
    idx = np.arange(1, w.size + 1, dtype=np.uint64)
    with np.errstate(over="ignore"):
        keys = idx * np.uint64(0x9E3779B97F4A7C15) + np.uint64(seed & 0xFFFFFFFFFFFFFFFF)
        total = np.sum(_fmix64(w ^ keys), dtype=np.uint64)
    return int(total)


def as_u64(x: int) -> int:
    return x & 0xFFFFFFFFFFFFFFFF
