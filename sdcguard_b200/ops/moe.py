"""Grouping of mixture-of-experts rows for the grouped checked GEMM (`csrc/moe.cu`), all on the device:

    grp = Grouping(max_tokens, top_k, experts, hidden, device)
    xg, row_sq = grp.group(x, ids)                 # rows grouped by expert on 128-row bands, pads zeroed
    h = gemm.checked_linear_grouped(xg, w13, grp.gband, grp.gcount, state, slot, row_sq=row_sq)
    ...
    y = grp.combine(yg, wts)                        # y[t] = sum_k w[t, k] yg[row(t, k)], fp32, k order

No call reads anything back to the host, so a layer of these launches can be captured in a CUDA graph. The
capacity of the grouped buffers is tokens x top-k + experts x 127 rows, rounded up to whole bands: every routing
fits.

Reference: the expert GEMMs the reference checks are vLLM's fused MoE (src/sdcguard/serve_moe.py:123-165) and
PyTorch's `_grouped_mm`, per group (src/sdcguard/guard.py:102-143).
"""
from __future__ import annotations

from typing import Optional

import torch

from .. import _native

BAND = 128


def _s(dev) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def capacity(tokens: int, top_k: int, experts: int) -> int:
    """Rows of the grouped buffers that hold any routing of `tokens` tokens."""
    return -(-(tokens * top_k + experts * (BAND - 1)) // BAND) * BAND


class Grouping:
    def __init__(self, max_tokens: int, top_k: int, experts: int, hidden: int, device, e_lo: int = 0):
        """experts: the local experts e_lo .. e_lo + experts - 1 (pairs routed elsewhere are skipped)."""
        self.T, self.k, self.E, self.H, self.e_lo = max_tokens, top_k, experts, hidden, e_lo
        dev = self.device = torch.device(device)
        self.cap = capacity(max_tokens, top_k, experts)
        i32 = dict(dtype=torch.int32, device=dev)
        self.pos = torch.empty(max_tokens * top_k, **i32)
        self.offs = torch.zeros(experts + 1, **i32)
        self.cnt = torch.zeros(experts, **i32)
        self.gband = torch.zeros(self.cap // BAND, **i32)
        self.gcount = torch.zeros(1, **i32)
        self.err = torch.zeros(1, **i32)
        self.xg = torch.zeros(self.cap, hidden, dtype=torch.bfloat16, device=dev)
        self.row_sq = torch.zeros(self.cap, dtype=torch.float32, device=dev)
        self.tokens = 0

    def group(self, x: torch.Tensor, ids: torch.Tensor):
        """x (T, H) bf16, ids (T, k) int32 -> (grouped rows (cap, H), their sums of squares (cap,))."""
        T = x.shape[0]
        if T > self.T or ids.shape != (T, self.k):
            raise ValueError(f"{T} tokens x {tuple(ids.shape)} ids exceed the grouping ({self.T} x {self.k})")
        if x.dtype != torch.bfloat16 or x.stride(1) != 1 or x.shape[1] != self.H:
            raise ValueError("x must be (T, hidden) bf16 with unit column stride")
        self.tokens = T
        lib = _native.lib()
        ids = ids.contiguous()
        s = _s(self.device)
        _native.check(lib.sdc_moe_plan(ids.data_ptr(), T * self.k, self.e_lo, self.E, self.cap, self.pos.data_ptr(),
                                       self.offs.data_ptr(), self.cnt.data_ptr(), self.gband.data_ptr(),
                                       self.gcount.data_ptr(), self.err.data_ptr(), s), "moe plan")
        _native.check(lib.sdc_moe_gather(x.data_ptr(), x.stride(0), self.H, self.k, T * self.k, self.E,
                                         self.pos.data_ptr(), self.offs.data_ptr(), self.cnt.data_ptr(),
                                         self.xg.data_ptr(), self.row_sq.data_ptr(), s), "moe gather")
        return self.xg, self.row_sq

    def combine(self, yg: torch.Tensor, wts: torch.Tensor, out: Optional[torch.Tensor] = None,
                accumulate: bool = False) -> torch.Tensor:
        """yg (cap, H') grouped expert outputs, wts (T, k) fp32 -> (T, H') bf16 (added to `out` when
        accumulate)."""
        T, Hy = self.tokens, yg.shape[1]
        if out is None:
            out = torch.empty(T, Hy, dtype=torch.bfloat16, device=yg.device)
        wts = wts.contiguous().float()
        _native.check(_native.lib().sdc_moe_combine(yg.data_ptr(), Hy, T, self.k, self.pos.data_ptr(),
                                                    wts.data_ptr(), out.data_ptr(), out.stride(0), int(accumulate),
                                                    _s(yg.device)), "moe combine")
        return out

    def expert_rows(self) -> list:
        """Host copy of each local expert's (first row, rows) (diagnostics and tests; reads the device)."""
        offs, cnt = self.offs.tolist(), self.cnt.tolist()
        return [(offs[e], cnt[e]) for e in range(self.E)]
