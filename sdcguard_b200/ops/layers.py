"""Python entry points of the layer kernels in `csrc/layers.cu` and the exact replay comparison in
`csrc/checks.cu`. All take bf16 CUDA tensors and run on the current stream; optional `rows` index tensors
(int32, on the device) select rows for a replay of sampled rows."""
from __future__ import annotations

from typing import Optional

import torch

from .. import _native


def _s(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _p(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def add_rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, residual: Optional[torch.Tensor] = None,
                resid_out: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                row_sq: Optional[torch.Tensor] = None, rows: Optional[torch.Tensor] = None,
                check: Optional[torch.Tensor] = None):
    """y = RMSNorm(x (+ residual)) * weight; h = x + residual written to resid_out (may alias residual);
    ||y_row||^2 to row_sq. Returns (y, row_sq). With `rows`, output row i is computed from input row rows[i].
    With `check` (a state row) and `rows`: replay check, rows rows[i] of `out` (the first run's output) are
    recomputed and compared, nothing is written."""
    m = x.shape[0] if rows is None else rows.shape[0]
    h = x.shape[-1]
    if out is None:
        out = torch.empty(m, h, dtype=torch.bfloat16, device=x.device)
    if row_sq is None and check is None:
        row_sq = torch.empty(m, dtype=torch.float32, device=x.device)
    _native.check(_native.lib().sdc_add_rmsnorm_bf16(
        x.data_ptr(), _p(residual), weight.data_ptr(), float(eps), m, h, out.data_ptr(), _p(resid_out),
        _p(row_sq), _p(rows), _p(check), _s(x)), "add_rmsnorm")
    return out, row_sq


def qk_norm_rope_kv(qkv: torch.Tensor, nq: int, nkv: int, pos: torch.Tensor, slots: torch.Tensor,
                    q_norm: Optional[torch.Tensor], k_norm: Optional[torch.Tensor], eps: float,
                    cos_sin: torch.Tensor, q_out: torch.Tensor, cache: torch.Tensor,
                    rows: Optional[torch.Tensor] = None, check: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Split the fused QKV output, per-head RMSNorm of q and k (when weights are given), RoPE, q -> q_out,
    k/v -> paged cache at `slots` (int64; -1 skips). With `check` (a state row), compare instead of write."""
    t = qkv.shape[0] if rows is None else rows.shape[0]
    _native.check(_native.lib().sdc_qk_norm_rope_kv(
        qkv.data_ptr(), qkv.stride(0), t, nq, nkv, 128, pos.data_ptr(), slots.data_ptr(), _p(q_norm), _p(k_norm),
        float(eps), cos_sin.data_ptr(), q_out.data_ptr(), cache.data_ptr(), _p(rows), _p(check), _s(qkv)),
        "qk_norm_rope_kv")
    return q_out


def silu_mul(gu: torch.Tensor, out: Optional[torch.Tensor] = None, row_sq: Optional[torch.Tensor] = None,
             rows: Optional[torch.Tensor] = None, check: Optional[torch.Tensor] = None):
    """out = silu(gate) * up with ||out_row||^2; `rows` / `check` as in add_rmsnorm (replay check in place)."""
    m = gu.shape[0] if rows is None else rows.shape[0]
    i = gu.shape[-1] // 2
    if out is None:
        out = torch.empty(m, i, dtype=torch.bfloat16, device=gu.device)
    if row_sq is None and check is None:
        row_sq = torch.empty(m, dtype=torch.float32, device=gu.device)
    _native.check(_native.lib().sdc_silu_mul_bf16(gu.data_ptr(), m, i, out.data_ptr(), _p(row_sq), _p(rows),
                                                   _p(check), _s(gu)), "silu_mul")
    return out, row_sq


def silu_mul_bands(gu: torch.Tensor, gcount: torch.Tensor, out: Optional[torch.Tensor] = None,
                   row_sq: Optional[torch.Tensor] = None):
    """silu_mul over grouped expert rows: only the first 128 * gcount rows (gcount on the device) are computed."""
    m, i = gu.shape[0], gu.shape[-1] // 2
    if out is None:
        out = torch.empty(m, i, dtype=torch.bfloat16, device=gu.device)
    if row_sq is None:
        row_sq = torch.empty(m, dtype=torch.float32, device=gu.device)
    _native.check(_native.lib().sdc_silu_mul_bf16_bands(gu.data_ptr(), m, i, out.data_ptr(), row_sq.data_ptr(),
                                                        gcount.data_ptr(), _s(gu)), "silu_mul (bands)")
    return out, row_sq


def compare_rows(a: torch.Tensor, idx: Optional[torch.Tensor], b: torch.Tensor, state_row: torch.Tensor) -> None:
    """Exact comparison of replayed rows b[i] with a[idx[i]] (2-D bf16); mismatches go to `state_row`."""
    s = b.shape[0]
    _native.check(_native.lib().sdc_compare_rows_bf16(
        a.data_ptr(), a.stride(0), _p(idx), b.data_ptr(), b.stride(0), a.shape[-1], s, state_row.data_ptr(), _s(a)),
        "compare_rows")


def rope_table(max_pos: int, head_dim: int, theta: float, scaling: Optional[dict] = None,
               device="cuda") -> torch.Tensor:
    """(max_pos, head_dim / 2) float2 table of (cos, sin) for the rotate-half RoPE; `scaling` follows the
    Llama-3 frequency rule (factor, low_freq_factor, high_freq_factor, original_max_position_embeddings)."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    if scaling:
        import math
        factor = scaling["factor"]
        lo, hi = scaling["low_freq_factor"], scaling["high_freq_factor"]
        old = scaling["original_max_position_embeddings"]
        lo_wl, hi_wl = old / lo, old / hi
        wl = 2 * math.pi / inv
        smooth = (old / wl - lo) / (hi - lo)
        scaled = torch.where(wl > lo_wl, inv / factor, inv)
        mid = (wl <= lo_wl) & (wl >= hi_wl)
        inv = torch.where(mid, (1 - smooth) * inv / factor + smooth * inv, scaled)
    ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None, :]
    tab = torch.stack([ang.cos(), ang.sin()], dim=-1).float()
    return tab.contiguous().to(device)
