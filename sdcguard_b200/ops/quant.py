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

Zero points, three readings of one formula (`zero_mode`):
  "subtract"       W = rnd((q - z) s)                 Marlin: q - z is an exact small integer, one rounding
  "fma"            W = rnd(q s + zs), zs = -rnd(s z)  a fused multiply-add over a zero term rounded at load
  "two_roundings"  W = rnd(rnd(q s) + zs)             the same as two separately rounded steps
In float32, q s (an integer below 256 times an 8-bit significand) and q s + zs (under 2^17 units of the scale's last
place) are exact, so each reading costs one or two explicit roundings and nothing else. Which one a kernel uses is
a compiler decision for some kernels, so `probe()` decides: it runs the kernel on unit vectors, whose products are
the columns of W exactly (one product by 1.0 per output, added to zeros in fp32), and compares bit for bit.

`from_vllm(layer, kernel)` reads a vLLM mixed-precision linear layer (its kernel's parameter names and config;
the parameters' input / output / packed dimensions) before the kernel repacks the weights: int32 words holding
32 / bits codes each, lowest bits first, along the packed dimension. Layers with activation reordering (g_idx) or
one scale per output column (the scale applied after the accumulation, a second rounding) raise `Unsupported`.

Reference: src/sdcguard/_quant.py:1-60 (the effective weights of vLLM's Marlin and Machete layers and their checks),
`from_layer` :232, `probe` :278.
"""
from __future__ import annotations

from typing import Optional

import torch

from .. import _native
from . import gemm


ZERO_MODES = ("subtract", "fma", "two_roundings")


class Unsupported(ValueError):
    """A quantized layer whose arithmetic this module does not restate (the reason is the message)."""


class QuantWeights:
    def __init__(self, codes: torch.Tensor, scales: torch.Tensor, zeros: Optional[torch.Tensor], bits: int,
                 group: int, k: Optional[int] = None, zero_mode: str = "subtract"):
        """codes: uint8 [n, k / 2] (INT4, low nibble first) or [n, k] (INT8); scales: bf16 [n, k / group]; zeros:
        uint8 [n, k / group] or None (symmetric: zero point 8 for INT4, 128 for INT8)."""
        if bits not in (4, 8):
            raise ValueError("bits must be 4 or 8")
        if zero_mode not in ZERO_MODES:
            raise ValueError(f"zero_mode must be one of {ZERO_MODES}")
        self.zero_mode = zero_mode
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

    @classmethod
    def from_codes(cls, q: torch.Tensor, scales: torch.Tensor, zeros: Optional[torch.Tensor], bits: int, group: int,
                   zero_mode: str = "subtract") -> "QuantWeights":
        """From unpacked integer codes q [n, k] (values 0 .. 2^bits - 1), scales [n, k / group] and zero-point codes
        [n, k / group] (or None)."""
        q = q.to(torch.uint8)
        codes = (q[:, 0::2] | (q[:, 1::2] << 4)).contiguous() if bits == 4 else q.contiguous()
        return cls(codes, scales.to(torch.bfloat16).contiguous(),
                   None if zeros is None else zeros.to(torch.uint8).contiguous(), bits, group, q.shape[1], zero_mode)

    def with_zero_mode(self, mode: str) -> "QuantWeights":
        return QuantWeights(self.codes, self.scales, self.zeros, self.bits, self.group, self.k, mode)

    def effective_weight(self) -> torch.Tensor:
        """W (n, k) bf16 on the codes' device: the matrix the quantized GEMM multiplies by (`zero_mode`)."""
        if self.zero_mode != "subtract" and self.zeros is not None:
            return self._zero_term_weight(self.codes.device)
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

    def _zero_term_weight(self, device) -> torch.Tensor:
        """The "fma" and "two_roundings" readings on `device`, in float32 (exact before each explicit rounding)."""
        g = self.group
        q = self._codes_unpacked().to(device).float()
        s = self.scales.to(device).float().repeat_interleave(g, dim=1)
        zs = -(self.scales.to(device).float() * self.zeros.to(device).float()).to(torch.bfloat16).float()
        zs = zs.repeat_interleave(g, dim=1)
        qs = q * s
        if self.zero_mode == "two_roundings":
            qs = qs.to(torch.bfloat16).float()
        return (qs + zs).to(torch.bfloat16)

    def reference_weight(self) -> torch.Tensor:
        """float64 restatement of the effective weight, rounded to bf16 (as float64), on the CPU."""
        q = self._codes_unpacked().double()
        s = self.scales.cpu().double().repeat_interleave(self.group, dim=1)
        if self.zeros is not None and self.zero_mode != "subtract":
            zs = -(self.scales.cpu().double() * self.zeros.cpu().double()).to(torch.bfloat16).double()
            qs = q * s
            if self.zero_mode == "two_roundings":
                qs = qs.to(torch.bfloat16).double()
            return (qs + zs.repeat_interleave(self.group, dim=1)).to(torch.bfloat16).double()
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


# ------------------------------------------------------------------------------------------ vLLM layers
def unpack_words(t: torch.Tensor, bits: int, axis: int) -> torch.Tensor:
    """int32 words holding 32 / bits codes each, lowest bits first, along `axis` -> int32 codes (that axis grows by
    32 / bits)."""
    per = 32 // bits
    w = t.to(torch.int64) & 0xFFFFFFFF
    shifts = torch.arange(per, device=t.device, dtype=torch.int64) * bits
    codes = (w.unsqueeze(-1) >> shifts) & ((1 << bits) - 1)           # [..., per] beside the last dim
    codes = codes.movedim(-1, axis + 1)                                 # per right after the packed axis
    shape = list(t.shape)
    shape[axis] *= per
    return codes.reshape(shape).to(torch.int32)


def _dims(p: torch.Tensor) -> tuple:
    """(input dim, output dim) of a 2-D vLLM parameter (one may be implied by the other)."""
    i, o = getattr(p, "input_dim", None), getattr(p, "output_dim", None)
    if i is None and o is None:
        raise Unsupported("parameter without input / output dimensions")
    if i is None:
        i = 1 - o
    if o is None:
        o = 1 - i
    return i, o


def _as_n_by(p: torch.Tensor, data: torch.Tensor) -> torch.Tensor:
    """data laid out like p (same input / output dims) as [output, input]."""
    i, o = _dims(p)
    return data if (o, i) == (0, 1) else data.t()


def from_vllm(layer: torch.nn.Module, kernel) -> QuantWeights:
    """The effective weights of a vLLM mixed-precision linear layer, read before `kernel` repacks them (see the
    module docstring). `kernel` carries `config` (weight_type, group_size, zero_points, has_g_idx,
    partition_weight_shape) and the parameter names `w_q_name`, `w_s_name`, `w_zp_name`, `w_gidx_name`."""
    c = kernel.config
    act = getattr(c, "act_type", None)
    if isinstance(act, torch.dtype) and act.itemsize == 1:
        raise Unsupported(f"activations quantized to {act} inside the kernel (weight-only layers only)")
    wt = c.weight_type
    bits = int(wt.size_bits)
    if bits not in (4, 8) or not getattr(wt, "is_integer", lambda: True)():
        raise Unsupported(f"weight type {wt} (INT4 and INT8 codes only)")
    if c.has_g_idx:
        g = getattr(layer, kernel.w_gidx_name or "", None)
        if g is not None and g.numel() and not torch.equal(g.cpu(), torch.arange(g.numel(), dtype=g.dtype) //
                                                               max(1, int(c.group_size))):
            raise Unsupported("activation reordering (g_idx)")
    k, n = (int(x) for x in c.partition_weight_shape)
    group = int(c.group_size)
    if group == -1:
        raise Unsupported("one scale per output column: the kernel applies it after accumulating (a second rounding)")
    wq = getattr(layer, kernel.w_q_name)
    pd = getattr(wq, "packed_dim", None)
    q = unpack_words(wq.data, bits, pd) if pd is not None and wq.dtype == torch.int32 else wq.data.to(torch.int32)
    q = _as_n_by(wq, q)
    if tuple(q.shape) != (n, k):
        raise Unsupported(f"codes {tuple(q.shape)} against the partition's (n, k) = {(n, k)}")
    ws = getattr(layer, kernel.w_s_name)
    scales = _as_n_by(ws, ws.data)
    zeros = None
    if c.zero_points:
        wz = getattr(layer, kernel.w_zp_name)
        zpd = getattr(wz, "packed_dim", None)
        z = unpack_words(wz.data, bits, zpd) if zpd is not None and wz.dtype == torch.int32 else wz.data
        zeros = _as_n_by(wz, z)[:, : scales.shape[1]]
        if zeros.shape[0] != n:
            zeros = zeros[:n]
    elif getattr(wt, "has_bias", lambda: False)() and int(wt.bias) != (8 if bits == 4 else 128):
        raise Unsupported(f"weight type {wt}: code offset {wt.bias}")
    if scales.dtype not in (torch.bfloat16, torch.float16) or tuple(scales.shape) != (n, k // group):
        raise Unsupported(f"scales {scales.dtype} {tuple(scales.shape)}")
    mode = "fma" if zeros is not None and "machete" in type(kernel).__name__.lower() else "subtract"
    return QuantWeights.from_codes(q, scales, zeros, bits, group, mode)


def probe_columns(k: int, group: int, limit: int = 256, seed: int = 0) -> list:
    """Input positions to probe: the first and last of every group (where its scale and zero point start and end),
    evenly thinned to `limit`, or topped up with random positions to `limit`."""
    import random
    edges = sorted({c for g in range(0, k, group) for c in (g, min(k, g + group) - 1)})
    if len(edges) >= limit:
        step = len(edges) / limit
        return sorted({edges[int(i * step)] for i in range(limit)})
    taken = set(edges)
    rest = [c for c in range(k) if c not in taken]
    random.Random(seed).shuffle(rest)
    return sorted(edges + rest[:limit - len(edges)])


def probe(apply, w_eff: torch.Tensor, cols, dtype=torch.bfloat16) -> dict:
    """Run a quantized kernel (`apply(x)`, x [m, k]) on unit vectors e_c for c in cols: its output row for e_c is
    column c of the matrix it multiplies by, exactly. Compared bit for bit with w_eff [n, k]."""
    cols = list(cols)
    x = torch.zeros(len(cols), w_eff.shape[1], dtype=dtype, device=w_eff.device)
    x[torch.arange(len(cols)), torch.tensor(cols)] = 1
    y = apply(x).to(torch.bfloat16)
    want = w_eff[:, cols].t().to(torch.bfloat16)
    bad = (y.view(torch.int16) != want.view(torch.int16))
    nbad = int(bad.sum().item())
    first = None
    if nbad:
        r, j = (int(v) for v in bad.nonzero()[0].tolist())
        first = {"input": cols[r], "output": j, "kernel": float(y[r, j]), "restated": float(want[r, j])}
    return {"ok": nbad == 0, "columns": len(cols), "mismatches": nbad, "first": first}
