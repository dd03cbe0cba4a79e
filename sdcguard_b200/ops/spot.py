"""Sampled exact check of a linear layer's outputs (`csrc/spot.cu`): a few (row, column) outputs of y = x W^T
(+ bias) recomputed exactly and compared with the stored bf16 value against a per-output bound.

    sched = SpotSchedule(n_cols=w.shape[0])
    rows, cols = sched.sample(m, turn)                   # device int32 lists
    spot_check(x, w, y, rows, cols, state_row, bias)     # alarms go into the layer's state row (line 6)

Why it exists beside the ABFT check: the ABFT check judges a 128-column block against that block's noise, so it
misses a change to one output that is small next to the block (a low mantissa bit of an output near zero); this
check judges each sampled output against its own magnitude. It sees few outputs per call, so it runs on a rotating
sample (columns walk the layer with a golden-ratio stride, rows spread over the batch and move each turn).

Reference: `SpotChecks` (src/sdcguard/serve_spot.py:639), `col_step` (:168), bound (:1-56).
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from .. import _native
from ..numerics import abft

SPOT_COLS = 8
SPOT_ROWS = 32


def _coprime_step(n: int) -> int:
    """A stride near n / golden ratio that is coprime with n, so the column walk visits every column."""
    if n <= 1:
        return 1
    s = max(1, int(round(n / ((1 + 5 ** 0.5) / 2))))
    while math.gcd(s, n) != 1:
        s += 1
    return s


class SpotSchedule:
    """Which outputs of a layer (n_cols wide) a turn looks at: SPOT_COLS columns evenly spread, offset by a
    golden-ratio walk, and up to SPOT_ROWS rows evenly spread over the batch, shifted by one each turn."""

    def __init__(self, n_cols: int, n_spot_cols: int = SPOT_COLS, n_spot_rows: int = SPOT_ROWS):
        self.n = n_cols
        self.c = min(n_spot_cols, n_cols)
        self.r = n_spot_rows
        self.step = _coprime_step(n_cols)

    def columns(self, turn: int) -> list[int]:
        off = (turn * self.step) % self.n
        gap = self.n // self.c
        return [(off + i * gap) % self.n for i in range(self.c)]

    def rows(self, m: int, turn: int) -> list[int]:
        if m <= self.r:
            return list(range(m))
        gap = m / self.r
        return sorted({(int(i * gap) + turn) % m for i in range(self.r)})

    def sample(self, m: int, turn: int, device) -> tuple[torch.Tensor, torch.Tensor]:
        r = torch.tensor(self.rows(m, turn), dtype=torch.int32)
        c = torch.tensor(self.columns(turn), dtype=torch.int32)
        return r.to(device, non_blocking=True), c.to(device, non_blocking=True)


def coefficients(k: int, c1: float = abft.C1, c2: float = abft.C2, c3: float = abft.C3,
                 nfma: int = abft.NFMA) -> tuple[float, float]:
    """(c1 sqrt(K), c2 sqrt(K) + c3 K / nfma + 1): the accumulation allowance of the bound for inner size K."""
    sk = math.sqrt(k)
    return c1 * sk, c2 * sk + (c3 * k / nfma if nfma else 0.0) + 1.0


def spot_check(x: torch.Tensor, w: torch.Tensor, y: torch.Tensor, rows: torch.Tensor, cols: torch.Tensor,
               state_row: torch.Tensor, bias: Optional[torch.Tensor] = None, c1: float = abft.C1,
               c2: float = abft.C2, c3: float = abft.C3) -> None:
    """x (m, k) bf16, w (n, k) bf16 contiguous, y (m, n) bf16 the layer's stored output, bias (n) fp32 or None;
    rows / cols int32 on the device; state_row int64 [4] (a StateTable row)."""
    if x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16 or y.dtype != torch.bfloat16:
        raise ValueError("spot_check takes bf16 x, w and y")
    if x.stride(1) != 1 or not w.is_contiguous() or y.stride(1) != 1:
        raise ValueError("spot_check needs unit column strides and a contiguous weight")
    n, k = w.shape
    a1, a2 = coefficients(k, c1, c2, c3)
    b = None if bias is None else bias.float().contiguous()
    _native.check(_native.lib().sdc_spot_check(
        x.data_ptr(), x.stride(0), w.data_ptr(), y.data_ptr(), y.stride(0), None if b is None else b.data_ptr(),
        n, k, rows.data_ptr(), rows.numel(), cols.data_ptr(), cols.numel(), float(a1), float(a2),
        state_row.data_ptr(), torch.cuda.current_stream(x.device).cuda_stream), "spot check")


def reference_scores(x: torch.Tensor, w: torch.Tensor, y: torch.Tensor, bias: Optional[torch.Tensor] = None,
                     c1: float = abft.C1, c2: float = abft.C2, c3: float = abft.C3) -> torch.Tensor:
    """Every output's spot score in float64 (the kernel's bound; for tests): (m, n)."""
    xd, wd = x.double(), w.double()
    r = xd @ wd.t()
    if bias is not None:
        r = r + bias.double()[None, :]
    a1, a2 = coefficients(w.shape[1], c1, c2, c3)
    norms = xd.norm(dim=1)[:, None] * wd.norm(dim=1)[None, :]
    bound = 2.0 ** -8 * r.abs() + 6 * 2.0 ** -24 * (a1 * norms + a2 * r.abs()) + 1e-30
    return (y.double() - r).abs() / bound
