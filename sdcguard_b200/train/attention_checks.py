"""Identity checks of fused attention in training, which no GEMM checksum covers (the fused kernel never exposes
its matmuls):

  * forward: every output o[q, d] is a convex combination of v[k, d] over the attended keys, so it lies within
    [min_k v[k, d], max_k v[k, d]] (up to the output rounding);
  * backward: dV = P^T dO and every row of P sums to 1, so sum_k dV[k, d] = sum_q dO[q, d] for each head (with
    grouped-query attention, summed over the heads that share a kv head).

Both return the worst score (excess over the rounding bound, in units of it); a score above 6 is an alarm.

Reference: `forward_stat` / `backward_stat` (src/sdcguard/attention.py:114, :171).
"""
from __future__ import annotations

import torch

U_BF16 = 2.0 ** -8
U_F16 = 2.0 ** -11
U_F32 = 2.0 ** -24


def _unit(dtype) -> float:
    return {torch.bfloat16: U_BF16, torch.float16: U_F16}.get(dtype, U_F32)


def forward_stat(o: torch.Tensor, v: torch.Tensor) -> float:
    """o: (B, Hq, T, D), v: (B, Hkv, S, D) (all keys attendable: the bound uses the full key range, which any
    mask only narrows). Returns the worst excess over [min v, max v] in units of the rounding bound."""
    B, Hq, T, D = o.shape
    g = Hq // v.shape[1]
    vf = v.float()
    lo = vf.amin(dim=2).repeat_interleave(g, dim=1)[:, :, None, :]     # (B, Hq, 1, D)
    hi = vf.amax(dim=2).repeat_interleave(g, dim=1)[:, :, None, :]
    of = o.float()
    span = torch.maximum(hi.abs(), lo.abs())
    bound = 2 * _unit(o.dtype) * span + 1e-30
    excess = torch.clamp(of - hi, min=0) + torch.clamp(lo - of, min=0)
    return float((excess / bound).max())


def backward_stat(dv: torch.Tensor, do: torch.Tensor) -> float:
    """dv: (B, Hkv, S, D), do: (B, Hq, T, D). sum over keys of dV equals sum over queries of dO per kv head."""
    B, Hkv, S, D = dv.shape
    Hq, T = do.shape[1], do.shape[2]
    g = Hq // Hkv
    lhs = dv.double().sum(dim=2)                                          # (B, Hkv, D)
    rhs = do.double().view(B, Hkv, g, T, D).sum(dim=(2, 3))               # (B, Hkv, D)
    mag = dv.double().abs().sum(dim=2) + do.double().abs().view(B, Hkv, g, T, D).sum(dim=(2, 3))
    u = max(_unit(dv.dtype), _unit(do.dtype))
    bound = u * mag * (S + T) ** 0.5 + 1e-30
    return float(((lhs - rhs).abs() / bound).max())
