"""Weight-only quantized linear layers (INT4 / INT8 codes with group scales, optional zero points), checked.

    qw = QuantWeights.quantize(w, bits=4, group=128)     # or QuantWeights(codes, scales, zeros, bits, group)
    layer = CheckedQuantLinear(qw)
    y = layer(x, state, slot)                             # the checked GEMM on the layer's effective weights

A weight-only GEMM dequantizes each weight into bf16 before its fp32 accumulation, so the matrix it multiplies by
is the effective weight W = rnd((q - z) s) (z: the group's zero point, or 8 / 128 for the symmetric formats), exact
in bf16. `effective_weight()` builds W on the device (`csrc/quant.cu`, one rounding per element, the same
arithmetic), the checksum rows come from W, and the checked tcgen05 GEMM multiplies by W: outputs and checks are
those of the layer's arithmetic. The GEMM reads W in bf16 (built once at load and kept), so this path checks
quantized layers but does not save their memory at run time; a main loop that expands the codes in shared memory
is not built.

`fingerprint()` hashes the codes, scales and zero points (the tensors a quantized kernel reads), so a weight scan
can find a change in the packed weights themselves; `reference_weight()` is the float64 CPU restatement used as the
test oracle.

Reference: src/sdcguard/_quant.py:1-60 (the effective weights of vLLM's Marlin and Machete layers and their checks).
"""
from __future__ import annotations

from typing import Optional

import torch

from .. import _native
from . import gemm


class QuantWeights:
    def __init__(self, codes: torch.Tensor, scales: torch.Tensor, zeros: Optional[torch.Tensor], bits: int,
                 group: int, k: Optional[int] = None):
        """codes: uint8 [n, k / 2] (INT4, low nibble first) or [n, k] (INT8); scales: bf16 [n, k / group]; zeros:
        uint8 [n, k / group] or None (symmetric: zero point 8 for INT4, 128 for INT8)."""
        if bits not in (4, 8):
            raise ValueError("bits must be 4 or 8")
        self.codes, self.scales, self.zeros, self.bits, self.group = codes, scales, zeros, bits, group
        self.n = codes.shape[0]
        self.k = k if k is not None else codes.shape[1] * (2 if bits == 4 else 1)
        if self.k % group or scales.shape != (self.n, self.k // group):
            raise ValueError("scales must be [n, k / group]")
        self.center = 8 if bits == 4 else 128

    @classmethod
    def quantize(cls, w: torch.Tensor, bits: int = 4, group: int = 128, zero_points: bool = False) -> "QuantWeights":
        """Round-to-nearest group quantization of a weight (a test and example helper)."""
        n, k = w.shape
        wf = w.float().view(n, k // group, group)
        qmax = (1 << bits) - 1
        if zero_points:
            lo, hi = wf.amin(-1, keepdim=True), wf.amax(-1, keepdim=True)
            s = ((hi - lo) / qmax).clamp_min(1e-8).to(torch.bfloat16).float()
            z = torch.round(-lo / s).clamp(0, qmax)
            q = torch.round(wf / s + z).clamp(0, qmax)
            zeros = z.squeeze(-1).to(torch.uint8)
        else:
            c = 1 << (bits - 1)
            s = (wf.abs().amax(-1, keepdim=True) / (c - 1)).clamp_min(1e-8).to(torch.bfloat16).float()
            q = torch.round(wf / s + c).clamp(0, qmax)
            zeros = None
        q = q.view(n, k).to(torch.uint8)
        codes = (q[:, 0::2] | (q[:, 1::2] << 4)).contiguous() if bits == 4 else q.contiguous()
        return cls(codes, s.view(n, k // group).to(torch.bfloat16), zeros, bits, group, k)

    def effective_weight(self) -> torch.Tensor:
        """W (n, k) bf16 on the codes' device: rnd((q - z) s), the matrix the quantized GEMM multiplies by."""
        if not self.codes.is_cuda:
            return self.reference_weight().to(torch.bfloat16)
        w = torch.empty(self.n, self.k, dtype=torch.bfloat16, device=self.codes.device)
        _native.check(_native.lib().sdc_dequant_weights(
            self.codes.data_ptr(), self.bits, self.n, self.k, self.group, self.scales.data_ptr(),
            None if self.zeros is None else self.zeros.data_ptr(), self.center, w.data_ptr(),
            torch.cuda.current_stream(self.codes.device).cuda_stream), "dequantize weights")
        return w

    def _codes_unpacked(self) -> torch.Tensor:
        c = self.codes.cpu()
        if self.bits == 8:
            return c.to(torch.int32)
        q = torch.empty(self.n, self.k, dtype=torch.int32)
        q[:, 0::2] = (c & 0xF).to(torch.int32)
        q[:, 1::2] = (c >> 4).to(torch.int32)
        return q

    def reference_weight(self) -> torch.Tensor:
        """float64 (q - z) s rounded to bf16 (as float64), on the CPU."""
        q = self._codes_unpacked().double()
        s = self.scales.cpu().double().repeat_interleave(self.group, dim=1)
        z = (self.zeros.cpu().double().repeat_interleave(self.group, dim=1) if self.zeros is not None
             else torch.full_like(q, float(self.center)))
        return ((q - z) * s).to(torch.bfloat16).double()

    def fingerprint(self) -> torch.Tensor:
        from .fingerprint import fingerprint
        ts = [self.codes, self.scales] + ([self.zeros] if self.zeros is not None else [])
        return fingerprint(ts)


class CheckedQuantLinear:
    """A weight-only quantized linear layer on the checked GEMM (effective weights built once, with their
    checksum rows)."""

    def __init__(self, qw: QuantWeights, bias: Optional[torch.Tensor] = None):
        self.qw = qw
        self.cw = gemm.CheckedWeight(qw.effective_weight(), bias)
        self.codes_fp = qw.fingerprint()

    def __call__(self, x: torch.Tensor, state: torch.Tensor, slot: int, **kw) -> torch.Tensor:
        return gemm.checked_linear(x, self.cw, state, slot, **kw)

    def weights_unchanged(self) -> bool:
        """The packed codes, scales and zero points still hash to what they did at load (one device read)."""
        return bool(torch.equal(self.qw.fingerprint(), self.codes_fp))
