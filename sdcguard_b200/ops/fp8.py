"""Block-scaled fp8 checked GEMM (`csrc/gemm_fp8.cu`): E4M3 operands, 1 x 128 activation scales and 128 x 128 weight
scales (powers of two, as UE8M0 scale factors are), fp32 accumulation, bf16 output, ABFT check of every 128-column
block of every row in the same kernel.

    fw = Fp8Weight(w_bf16)                          # once: quantize W, checksum rows of the quantized blocks
    xq = quantize_act(x)                            # E4M3 codes, scales, ||dequantized row||^2
    y = checked_linear_fp8(xq, fw, state, slot)     # output + check
    quantize_act(x, out=xq, rows=sample, check=state[s])   # exact replay of sampled rows (quantisation check)

Checksum rows: for each 128-column block b of W and each 128-wide K block kb, the plain and the +-1-signed sums of
the block's quantized rows (sums of E4M3 values, exact in fp32) are split into six E4M3 parts, each with its own
power-of-two scale (`csc`), so 12 rows of fp8 carry about 24 significant bits; they are rows 16 b .. 16 b + 11 of
`wcq` (rows 12 to 15 zero) and ride in the same MMA as the tile's 128 weight rows.

Scale factors go to the tensor cores as UE8M0 bytes (the power-of-two scale 2^e is the byte e + 127) in 512-byte
chunks, one per 128 operand rows and 128-wide K block: row r at byte (r % 32) 16 + 4 (r // 32) + j for its four
32-wide K slices j (`sf_chunks`). The B operand of block b has two chunks per K block: its 128 weight rows (all the
block's scale) and its 16 checksum rows (part scale x block scale).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch

from .. import _native
from ..numerics import abft
from .gemm import _stream_ptr, error_word

FP8_MAX = 448.0
PARTS = 6


def pow2_scale(amax: torch.Tensor) -> torch.Tensor:
    """Smallest power of two s with amax / s <= 448 (1 where amax is 0)."""
    r = amax.double() / FP8_MAX
    m, e = torch.frexp(r)
    e = torch.where(m == 0.5, e - 1, e)
    s = torch.ldexp(torch.ones_like(r), e)
    return torch.where(amax > 0, s, torch.ones_like(r)).float()


def to_e4m3(x: torch.Tensor) -> torch.Tensor:
    return x.clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)


def ue8m0(s: torch.Tensor) -> torch.Tensor:
    """UE8M0 byte of power-of-two scales (2^e -> e + 127); 0 (an all-zero part) -> 127, i.e. 1.0."""
    s = s.float()
    b = (s.view(torch.int32) >> 23) & 0xFF
    return torch.where(s > 0, b, torch.full_like(b, 127)).to(torch.uint8)


def sf_chunks(sc: torch.Tensor) -> torch.Tensor:
    """(..., rows, kbs) scales of a 128 x rows-padded operand -> (..., ceil(rows / 128), kbs, 512) UE8M0 chunks."""
    *lead, rows, kbs = sc.shape
    t = -(-rows // 128)
    b = torch.full((*lead, t * 128, kbs), 127, dtype=torch.uint8, device=sc.device)
    b[..., :rows, :] = ue8m0(sc)
    n = len(lead)
    b = b.view(*lead, t, 4, 32, kbs)                                     # (..., t, r // 32, r % 32, kb)
    b = b.permute(*range(n), n, n + 3, n + 2, n + 1)                     # (..., t, kb, r % 32, r // 32)
    b = b.unsqueeze(-1).expand(*lead, t, kbs, 32, 4, 4)                  # (..., t, kb, r % 32, r // 32, j)
    return b.reshape(*lead, t, kbs, 512).contiguous()


class Fp8Weight:
    def __init__(self, weight: torch.Tensor, mask: Optional[tuple] = None, c1: float = abft.C1, c2: float = abft.C2,
                 c3: float = abft.C3):
        n, k = weight.shape
        if n % 128 or k % 128:
            raise ValueError(f"fp8 checked GEMM needs n and k multiples of 128 (got n={n}, k={k})")
        dev = weight.device
        self.n, self.k, self.nb, self.kbs = n, k, n // 128, k // 128
        self.mask = mask or abft.sign_mask()
        w = weight.detach().float().view(self.nb, 128, self.kbs, 128)
        self.sw = pow2_scale(w.abs().amax(dim=(1, 3))).contiguous()                  # (nb, kbs)
        q = to_e4m3(w / self.sw[:, None, :, None])
        self.wq = q.view(n, k).contiguous()
        qf = q.float()                                                                # quantized values
        deq = qf * self.sw[:, None, :, None]
        s = abft.sign_vector(self.mask, dtype=torch.float32, device=dev).view(1, 128, 1, 1)
        plain = qf.double().sum(1)                                                    # (nb, kbs, 128) exact
        signed = (qf.double() * s.double()).sum(1)
        rows = torch.zeros(self.nb, 16, self.kbs, 128, dtype=torch.float32, device=dev)
        csc = torch.zeros(self.nb, self.kbs, 12, dtype=torch.float32, device=dev)
        for j, total in enumerate((plain, signed)):
            r = total.clone()
            for i in range(PARTS):
                amax = r.abs().amax(dim=2)                                            # (nb, kbs)
                sc = pow2_scale(amax).double()
                part = to_e4m3((r / sc[..., None]).float()).float().double()
                rows[:, 6 * j + i] = part.float()
                csc[:, :, 6 * j + i] = torch.where(amax > 0, sc, torch.zeros_like(sc)).float()
                r = r - part * sc[..., None]
        self.wcq = to_e4m3(rows).view(self.nb * 16, self.kbs * 128).contiguous()
        self.csc = csc.contiguous()
        # scale-factor chunks of each block's 144-row B operand: 128 weight rows, 12 checksum parts, 116 unused. The
        # parts split sums of codes, so their scale factors are the part scale times the block's weight scale.
        bs = torch.zeros(self.nb, 256, self.kbs, dtype=torch.float32, device=dev)
        bs[:, :128] = self.sw[:, None, :]
        bs[:, 128:140] = (csc * self.sw[:, :, None]).transpose(1, 2)     # parts of sums of codes, times the block scale
        self.sfb = sf_chunks(bs).transpose(1, 2).reshape(self.nb, self.kbs, 1024).contiguous()
        dq = deq.view(self.nb, 128, k).double()
        pl, sg = dq.sum(1), (dq * s.view(1, 128, 1).double()).sum(1)
        self.wstat = torch.stack([torch.linalg.vector_norm(dq, dim=(1, 2)), torch.linalg.vector_norm(pl, dim=1),
                                  torch.linalg.vector_norm(sg, dim=1), dq.abs().amax(dim=(1, 2))], dim=1).float()
        self.prod_coef, self.out_coef = abft.coefficients(k, c1, c2, c3)

    def dequantized(self) -> torch.Tensor:
        return (self.wq.float().view(self.nb, 128, self.kbs, 128) * self.sw[:, None, :, None]).view(self.n, self.k)


@dataclass
class Fp8Act:
    q: torch.Tensor         # (m, k) float8_e4m3fn
    sa: torch.Tensor        # (m, k / 128) fp32 powers of two
    row_sq: torch.Tensor    # (m,) ||dequantized row||^2
    sf: torch.Tensor        # (ceil(m / 128), k / 128, 512) uint8 UE8M0 scale-factor chunks

    def dequantized(self) -> torch.Tensor:
        m, k = self.q.shape
        return (self.q.float().view(m, k // 128, 128) * self.sa[:, :, None]).view(m, k)


def quantize_act(x: torch.Tensor, out: Optional[Fp8Act] = None, rows: Optional[torch.Tensor] = None,
                 check: Optional[torch.Tensor] = None) -> Fp8Act:
    """x (m, k) bf16 -> E4M3 codes with 1 x 128 power-of-two scales. With rows and check: exact replay of the
    sampled rows against `out` (the stored codes and scales), nothing written."""
    m, k = x.shape
    if out is None:
        out = Fp8Act(torch.empty(m, k, dtype=torch.float8_e4m3fn, device=x.device),
                     torch.empty(m, k // 128, dtype=torch.float32, device=x.device),
                     torch.empty(m, dtype=torch.float32, device=x.device),
                     torch.full((-(-m // 128), k // 128, 512), 127, dtype=torch.uint8, device=x.device))
    _native.check(_native.lib().sdc_fp8_quant_act(
        x.data_ptr(), x.stride(0), m, k, out.q.data_ptr(), out.sa.data_ptr(), out.sf.data_ptr(), out.row_sq.data_ptr(),
        None if rows is None else rows.data_ptr(), 0 if rows is None else rows.numel(),
        None if check is None else check.data_ptr(), _stream_ptr(x.device)), "fp8 quantize")
    return out


def checked_linear_fp8(xa: Fp8Act, fw: Fp8Weight, state: torch.Tensor, slot: int, out: Optional[torch.Tensor] = None,
                       z_alarm: float = abft.Z_ALARM, inject: Optional[tuple] = None) -> torch.Tensor:
    m, k = xa.q.shape
    if k != fw.k:
        raise ValueError(f"activations have {k} columns, the weight {fw.k}")
    dev = xa.q.device
    if out is None:
        out = torch.empty(m, fw.n, dtype=torch.bfloat16, device=dev)
    s = fw.mask
    ir, ic, ix = (-1, -1, 0) if inject is None else (int(inject[0]), int(inject[1]), int(inject[2]))
    _native.check(_native.lib().sdc_gemm_fp8(
        xa.q.data_ptr(), xa.sf.data_ptr(), fw.wq.data_ptr(), fw.wcq.data_ptr(), fw.sfb.data_ptr(), m, fw.n, k, out.data_ptr(), out.stride(0), xa.row_sq.data_ptr(), fw.wstat.data_ptr(), state.data_ptr(),
        int(slot), s[0], s[1], s[2], s[3], float(z_alarm), float(fw.prod_coef), float(fw.out_coef),
        float(abft.ABS_FLOOR), float(math.sqrt(k)), error_word(dev).data_ptr(), ir, ic, ix, _stream_ptr(dev)),
        "fp8 checked GEMM")
    return out


class Fp8WeightStack:
    """The fp8-quantized weights of several experts (each (n, k), one shared sign pattern) stacked for
    `checked_linear_fp8_grouped`: codes (experts n, k), checksum rows (experts 16 n / 128, k), scale-factor chunks
    (experts n / 128, k / 128, 1024), block statistics (experts n / 128, 4)."""

    def __init__(self, weights: list, c1: float = abft.C1, c2: float = abft.C2, c3: float = abft.C3):
        if not weights:
            raise ValueError("Fp8WeightStack needs at least one weight")
        mask = abft.sign_mask()
        fws = [Fp8Weight(w, mask=mask, c1=c1, c2=c2, c3=c3) for w in weights]
        f0 = fws[0]
        if any((f.n, f.k) != (f0.n, f0.k) for f in fws):
            raise ValueError("expert weights must share one (n, k) shape")
        self.experts, self.n, self.k, self.nb, self.kbs, self.mask = len(fws), f0.n, f0.k, f0.nb, f0.kbs, mask
        self.wq = torch.cat([f.wq for f in fws]).contiguous()
        self.wcq = torch.cat([f.wcq for f in fws]).contiguous()
        self.sfb = torch.cat([f.sfb for f in fws]).contiguous()
        self.wstat = torch.cat([f.wstat for f in fws]).contiguous()
        self.prod_coef, self.out_coef = f0.prod_coef, f0.out_coef
        self.members = fws

    def expert(self, e: int) -> Fp8Weight:
        return self.members[e]


def checked_linear_fp8_grouped(xa: Fp8Act, stack: Fp8WeightStack, gband: torch.Tensor, gcount: torch.Tensor,
                               state: torch.Tensor, slot: int, out: Optional[torch.Tensor] = None,
                               z_alarm: float = abft.Z_ALARM, inject: Optional[tuple] = None) -> torch.Tensor:
    """The fp8 checked GEMM over every expert's rows in one launch: xa quantizes the grouped rows (expert rows on
    128-row tiles, ops.moe.Grouping or the expert-parallel receive), gband / gcount on the device."""
    m, k = xa.q.shape
    if k != stack.k:
        raise ValueError(f"activations have {k} columns, the weights {stack.k}")
    dev = xa.q.device
    if out is None:
        out = torch.empty(m, stack.n, dtype=torch.bfloat16, device=dev)
    s = stack.mask
    ir, ic, ix = (-1, -1, 0) if inject is None else (int(inject[0]), int(inject[1]), int(inject[2]))
    _native.check(_native.lib().sdc_gemm_fp8_grouped(
        xa.q.data_ptr(), xa.sf.data_ptr(), stack.wq.data_ptr(), stack.wcq.data_ptr(), stack.sfb.data_ptr(),
        stack.experts, m, stack.n, k, out.data_ptr(), out.stride(0), xa.row_sq.data_ptr(), stack.wstat.data_ptr(),
        gband.data_ptr(), gcount.data_ptr(), state.data_ptr(), int(slot), s[0], s[1], s[2], s[3], float(z_alarm),
        float(stack.prod_coef), float(stack.out_coef), float(abft.ABS_FLOOR), float(math.sqrt(k)),
        error_word(dev).data_ptr(), ir, ic, ix, _stream_ptr(dev)), "grouped fp8 checked GEMM")
    return out


class Fp8Linears:
    """The fp8 projections of a model: quantized weights by name, one activation scratch sized for the largest
    call (views keep their data pointers, so CUDA graphs can capture the calls), and the quantizer replay check."""

    def __init__(self, device):
        self.device = torch.device(device)
        self.weights: dict[str, Fp8Weight] = {}
        self.cap = (0, 0)
        self._q = self._sa = self._rs = self._sf = None

    def add(self, name: str, weight: torch.Tensor) -> Fp8Weight:
        fw = Fp8Weight(weight)
        self.weights[name] = fw
        return fw

    def reserve(self, rows: int, k: int) -> None:
        if rows * k <= self.cap[0] * self.cap[1] and rows <= self.cap[0]:
            return
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("fp8 activation scratch too small inside CUDA graph capture")
        rows, k = max(rows, self.cap[0]), max(k, self.cap[1])
        self._q = torch.empty(rows * k, dtype=torch.float8_e4m3fn, device=self.device)
        self._sa = torch.empty(rows * (k // 128), dtype=torch.float32, device=self.device)
        self._rs = torch.empty(rows, dtype=torch.float32, device=self.device)
        # bytes of rows past m are never written: 127 (1.0) keeps the padded MMA rows finite
        self._sf = torch.full((-(-rows // 128) * (k // 128) * 512,), 127, dtype=torch.uint8, device=self.device)
        self.cap = (rows, k)

    def act(self, m: int, k: int) -> Fp8Act:
        self.reserve(m, k)
        t = -(-m // 128)
        return Fp8Act(self._q[: m * k].view(m, k), self._sa[: m * (k // 128)].view(m, k // 128), self._rs[:m],
                      self._sf[: t * (k // 128) * 512].view(t, k // 128, 512))

    def linear(self, name: str, x: torch.Tensor, state: torch.Tensor, slot: int, out: torch.Tensor,
               qcheck: Optional[torch.Tensor] = None, sample: Optional[torch.Tensor] = None) -> torch.Tensor:
        m, k = x.shape
        xa = quantize_act(x, out=self.act(m, k))
        if qcheck is not None and sample is not None and sample.numel():
            quantize_act(x, out=xa, rows=sample, check=qcheck)
        return checked_linear_fp8(xa, self.weights[name], state, slot, out=out)
