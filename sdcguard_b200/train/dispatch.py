"""Operator-level training guard: a TorchDispatchMode that sees every aten matrix multiply of a step, forward and
backward (autograd's own matmuls included), with no change to the model.

    guard = DispatchGuard(check_every=10)
    for step, batch in enumerate(loader):
        with guard.at_step(step):               # active on steps where step % check_every == 0
            loss = model(batch).loss
            loss.backward()
        opt.step(); opt.zero_grad()
    guard.events, guard.coverage()

On an active step:
  mm, addmm (bf16 CUDA, alpha = beta = 1, 1-D bias, dimensions multiples of 8)
      run on this library's checked sm_100a GEMM: C = A B = A (B^T)^T with B^T materialised, the bias folded in,
      so the output carries the ABFT check of its fp32 accumulator (the check sits in the GEMM's epilogue).
      Checksum rows of a B operand are cached per storage and version for the step.
  every other mm, addmm, bmm, baddbmm, addbmm, mv, addmv and torch._grouped_mm in bf16, fp16 or fp32
      runs as PyTorch runs it and is then checked on the device: the plain and signed sums of every
      (batch, row, 128-column block) of the output against A times the block sums of B
      (`abft.product_zscores`), with the rounding of the output in the noise model; with precise=True the
      mm / addmm / bmm / baddbmm family keeps its fp32 accumulator (`aten.*.dtype`), is checked on it, and is
      rounded afterwards (the model sees the same rounding of the same fp32 result).
  scaled (fp8), integer and packed-weight matmuls are seen, counted and left unchecked, with their FLOPs.
Results fold into a device state table (no host synchronisation inside the step) and are read back once, when the
step's `with` block exits. While active, cuBLAS's reduced-precision split-K reductions are switched off (their
bf16 partial sums are outside the noise model) and restored on exit; unchecked steps are untouched.

This is the slow, model-agnostic mode; `SDCGuard.protect` (guard.py) is the fast one for nn.Linear.

Reference: src/sdcguard/guard.py:788 (`SDCGuard(TorchDispatchMode)`), :1651 (`__torch_dispatch__`), :222
(`matmul_checks`: the op table and how each op maps to A, B, C, bias, alpha, beta), :78-88 (the checked and the
counted-unchecked op sets), :146-215 (exact reductions on checked steps), :1420 (`at_step`), :1882 (read-back once
per step).
"""
from __future__ import annotations

import contextlib
from typing import Optional

import torch
from torch.utils._python_dispatch import TorchDispatchMode

from ..numerics import abft
from ..ops import gemm
from ..utils.events import EventLog, SDCEvent, device_identity
from .guard import SDCGuard

aten = torch.ops.aten

CHECKED = {"aten::mm", "aten::addmm", "aten::bmm", "aten::baddbmm", "aten::addbmm", "aten::mv", "aten::addmv",
           "aten::_grouped_mm"}
UNCHECKED = {"aten::_scaled_mm", "aten::_scaled_mm_v2", "aten::_scaled_grouped_mm", "aten::_scaled_grouped_mm_v2",
             "aten::_addmm_activation", "aten::_int_mm", "aten::_weight_int8pack_mm", "aten::_weight_int4pack_mm",
             "aten::_weight_int4pack_mm_with_scales_and_zeros"}
ROUND = {torch.bfloat16: 2.0 ** -8, torch.float16: 2.0 ** -11, torch.float32: 0.0}
CHUNK_BYTES = 256 << 20          # float64 working set of one product check


def _name(func) -> str:
    try:
        return func._schema.name
    except AttributeError:
        return str(func)


def _ab(args, kwargs, i: int, key: str, default=1):
    v = kwargs.get(key, args[i] if len(args) > i else default)
    return float(v)


class DispatchGuard(TorchDispatchMode):
    def __init__(self, check_every: int = 1, z_alarm: float = abft.Z_ALARM, device=None, precise: bool = False,
                 native_mm: bool = True, exact_reductions: bool = True, log: Optional[EventLog] = None,
                 on_alert=None):
        super().__init__()
        self.check_every = max(1, int(check_every))
        self.z_alarm = z_alarm
        self.device = torch.device(device if device is not None else ("cuda" if torch.cuda.is_available() else "cpu"))
        self.precise = precise
        self.native_mm = native_mm
        self.exact_reductions = exact_reductions
        self.table = gemm.StateTable(self.device, 256)
        self.slots: dict = {}
        self.log = log or EventLog()
        self.on_alert = on_alert
        self.events: list[SDCEvent] = []
        self.counts = {"native": 0, "checked": 0, "unchecked": 0, "checked_flops": 0, "unchecked_flops": 0}
        self.unchecked_ops: dict[str, int] = {}
        self.checks = 0
        self.unjudged = 0
        self.worst_clean = 0.0
        self._cw_cache: dict = {}
        self._mask = abft.sign_mask()
        self._inject: Optional[tuple] = None
        self._saved_flags = None

    # ---------------------------------------------------------------- schedule
    # the same schedule as SDCGuard: every N-th step, plus the windows of after_restart() and observe()
    should_check = SDCGuard.should_check
    after_restart = SDCGuard.after_restart
    observe = SDCGuard.observe

    @contextlib.contextmanager
    def on_step(self, step: int):
        """Wrap one training step: checked when should_check(step), otherwise untouched. Yields whether it is."""
        if self.should_check(step):
            with self.at_step(step, force=True):
                yield True
        else:
            yield False

    @contextlib.contextmanager
    def at_step(self, step: int, force: bool = False):
        if step % self.check_every and not force:
            yield self
            return
        self._cw_cache.clear()
        with self:
            yield self
        self.flush(step)

    def __enter__(self):
        if self.exact_reductions:
            m = torch.backends.cuda.matmul
            self._saved_flags = (m.allow_bf16_reduced_precision_reduction, m.allow_fp16_reduced_precision_reduction)
            m.allow_bf16_reduced_precision_reduction = False
            m.allow_fp16_reduced_precision_reduction = False
        return super().__enter__()

    def __exit__(self, *exc):
        try:
            return super().__exit__(*exc)
        finally:
            if self._saved_flags is not None:
                m = torch.backends.cuda.matmul
                m.allow_bf16_reduced_precision_reduction, m.allow_fp16_reduced_precision_reduction = self._saved_flags
                self._saved_flags = None

    def inject_next(self, row: int, col: int, bit: int, batch: int = 0) -> None:
        """Fault injection: the next checked matmul flips `bit` of its result at (batch, row, col): of the fp32
        accumulator on the native and precise paths, of the returned output otherwise (the model sees it too)."""
        self._inject = (batch, row, col, bit)

    # ---------------------------------------------------------------- dispatch
    def _slot(self, name: str, nb: int, kind: str) -> int:
        key = (name, nb, kind)
        if key not in self.slots:
            self.slots[key] = self.table.add(name, nb, kind)
        return self.slots[key]

    def __torch_dispatch__(self, func, types, args=(), kwargs=None):
        kwargs = kwargs or {}
        name = _name(func)
        if name in CHECKED and func._overloadname in ("default", ""):
            try:
                out = self._checked(name, func, args, kwargs)
            except _Skip:
                out = None
            if out is not None:
                return out
        out = func(*args, **kwargs)
        if name in CHECKED or name in UNCHECKED:
            self._count_unchecked(name, args, out)
        return out

    def _count_unchecked(self, name, args, out) -> None:
        self.counts["unchecked"] += 1
        self.unchecked_ops[name] = self.unchecked_ops.get(name, 0) + 1
        try:
            a = args[1] if name in ("aten::_addmm_activation", "aten::addmm", "aten::baddbmm", "aten::addbmm",
                                    "aten::addmv") else args[0]
            o = out[0] if isinstance(out, (tuple, list)) else out
            self.counts["unchecked_flops"] += 2 * int(o.numel()) * int(a.shape[-1])
        except Exception:  # noqa: BLE001 - counting only
            pass

    # Each op becomes one product A (G, m, k) @ B (G, k, n) = P, and the output out = beta * base + alpha * P.
    def _checked(self, name, func, args, kwargs):
        if name == "aten::mm":
            a, b = args[0], args[1]
            if self._native_ok(a, b, None):
                return self._native(name, a, b, None)
            return self._generic(name, func, args, kwargs, a, b, None, 1.0, 0.0, "mm")
        if name == "aten::addmm":
            base, a, b = args[0], args[1], args[2]
            beta, alpha = _ab(args, kwargs, 3, "beta"), _ab(args, kwargs, 4, "alpha")
            if beta == 1.0 and alpha == 1.0 and self._native_ok(a, b, base):
                return self._native(name, a, b, base)
            return self._generic(name, func, args, kwargs, a, b, base, alpha, beta, "addmm")
        if name == "aten::bmm":
            return self._generic(name, func, args, kwargs, args[0], args[1], None, 1.0, 0.0, "bmm")
        if name == "aten::baddbmm":
            beta, alpha = _ab(args, kwargs, 3, "beta"), _ab(args, kwargs, 4, "alpha")
            return self._generic(name, func, args, kwargs, args[1], args[2], args[0], alpha, beta, "baddbmm")
        if name == "aten::addbmm":
            b1, b2 = args[1], args[2]
            bb, m, k = b1.shape
            A = b1.permute(1, 0, 2).reshape(m, bb * k)                # sum_b b1[b] @ b2[b] = one matmul over k
            B = b2.reshape(bb * k, b2.shape[-1])
            beta, alpha = _ab(args, kwargs, 3, "beta"), _ab(args, kwargs, 4, "alpha")
            return self._generic(name, func, args, kwargs, A, B, args[0], alpha, beta, None)
        if name == "aten::mv":
            return self._generic(name, func, args, kwargs, args[0], args[1].unsqueeze(-1), None, 1.0, 0.0, None,
                                 vec=True)
        if name == "aten::addmv":
            beta, alpha = _ab(args, kwargs, 3, "beta"), _ab(args, kwargs, 4, "alpha")
            return self._generic(name, func, args, kwargs, args[1], args[2].unsqueeze(-1), args[0].unsqueeze(-1),
                                 alpha, beta, None, vec=True)
        if name == "aten::_grouped_mm":
            return self._grouped(func, args, kwargs)
        return None

    # ---- the native path: the checked tcgen05 GEMM
    def _native_ok(self, a, b, bias) -> bool:
        if not (self.native_mm and a.is_cuda and a.dtype == torch.bfloat16 and b.dtype == torch.bfloat16):
            return False
        if bias is not None and (bias.dim() != 1 or bias.dtype != torch.bfloat16):
            return False
        m, k = a.shape
        n = b.shape[1]
        return m > 0 and k % 8 == 0 and n % 8 == 0 and k > 0

    def _native(self, name, a, b, bias):
        m, k = a.shape
        n = b.shape[1]
        # Checksum rows are cached only for parameters (leaf tensors that require grad, or views of one): an
        # activation's storage can be freed and reused by another tensor of the same shape within the step.
        base = b._base if b._base is not None else b
        cache = base.is_leaf and base.requires_grad
        key = (b.untyped_storage().data_ptr(), b.storage_offset(), tuple(b.stride()), b._version,
               None if bias is None else (bias.data_ptr(), bias._version))
        cw = self._cw_cache.get(key) if cache else None
        if cw is None:
            w = b.t().contiguous()
            if w.data_ptr() % 16:
                w = w.clone()
            cw = gemm.CheckedWeight(w, None if bias is None else bias.float(), self._mask)
            if cache:
                self._cw_cache[key] = cw
        x = a.contiguous()
        if x.data_ptr() % 16 or x.stride(0) % 8:
            x = x.clone()
        slot = self._slot(f"{name} {m}x{k}x{n}", cw.nb, "gemm")
        inj = None
        if self._inject is not None:
            _, r, c, bit = self._inject
            self._inject = None
            inj = (r, c, 1 << bit)
        self.counts["native"] += 1
        self.counts["checked_flops"] += 2 * m * n * k
        return gemm.checked_linear(x, cw, self.table.state, slot, z_alarm=self.z_alarm, inject=inj)

    # ---- the library path: PyTorch's product, checked afterwards
    def _generic(self, name, func, args, kwargs, A, B, base, alpha, beta, acc_op, vec: bool = False):
        dt = A.dtype
        if dt not in ROUND or B.dtype != dt or A.device != B.device or A.shape[-1] == 0:
            raise _Skip
        if dt == torch.float32 and A.is_cuda and torch.backends.cuda.matmul.allow_tf32:
            raise _Skip                                    # TF32 products: outside the noise model
        if alpha == 0.0:
            raise _Skip
        precise = self.precise and acc_op is not None and dt != torch.float32
        if precise:
            P = self._acc(acc_op, A, B)                    # fp32 accumulator
            inj = self._take_inject()
            if inj is not None:
                _flip(P if P.dim() == 3 else P.unsqueeze(0), inj)
            outf = P if alpha == 1.0 else P * alpha
            if base is not None and beta != 0.0:
                outf = outf + beta * base.float()
            out = outf.to(dt)
            self._check(name, A, B, P, 0.0, None)
            return out
        out = func(*args, **kwargs)
        inj = self._take_inject()
        if inj is not None:
            o = out.unsqueeze(-1) if vec else out
            _flip(o if o.dim() == 3 else o.unsqueeze(0), inj)
        C = out.unsqueeze(-1) if vec else out
        judged = None
        if base is not None and beta != 0.0:
            bf = torch.broadcast_to(base, C.shape).double()
            Cf = (C.double() - beta * bf) / alpha
            judged = torch.isfinite(bf)
        else:
            Cf = C.double() / alpha if alpha != 1.0 else C
        self._check(name, A, B, Cf, ROUND[dt] / abs(alpha) if alpha != 1.0 else ROUND[dt], judged)
        return out

    def _acc(self, op, A, B):
        f = {"mm": aten.mm.dtype, "addmm": aten.mm.dtype, "bmm": aten.bmm.dtype, "baddbmm": aten.bmm.dtype}[op]
        if A.is_cuda:
            return f(A, B, torch.float32)
        return torch.matmul(A.float(), B.float())          # CPU: no out_dtype kernels; the fp32 product

    def _take_inject(self):
        inj, self._inject = self._inject, None
        return inj

    def _check(self, name, A, B, C, rnd, judged) -> None:
        """Queue the check of C ~ A @ B (2-D or batched) into the op's state row, on the device."""
        A3 = A if A.dim() == 3 else A.unsqueeze(0)
        B3 = B if B.dim() == 3 else B.unsqueeze(0)
        C3 = C if C.dim() == 3 else C.unsqueeze(0)
        G = max(A3.shape[0], B3.shape[0], C3.shape[0])
        m, k = A3.shape[1], A3.shape[2]
        n = B3.shape[2]
        A3, B3, C3 = A3.expand(G, m, k), B3.expand(G, k, n), C3.expand(G, m, n)
        if judged is not None:
            jb = judged if judged.dim() == 3 else judged.unsqueeze(0)
            jb = jb.expand(G, m, n)
        nb = -(-n // 128)
        if m == 0 or n == 0:
            return
        slot = self._slot(f"{name} {G}x{m}x{k}x{n}", nb, "rowblock")
        per_g = 8 * (m * k + k * nb * 128 + m * nb * 128 + 4 * m * nb)
        step = max(1, CHUNK_BYTES // max(per_g, 1))
        st = self.table.state[slot]
        for g0 in range(0, G, step):
            g1 = min(G, g0 + step)
            jz = None
            if judged is not None:
                jp = torch.nn.functional.pad(jb[g0:g1].logical_not(), (0, nb * 128 - n))
                jz = ~jp.view(g1 - g0, m, nb, 128).any(-1)
            z = abft.product_zscores(A3[g0:g1], B3[g0:g1], C3[g0:g1], self._mask, rnd_unit=rnd, judged=jz,
                                     z_alarm=self.z_alarm)
            flat = z.reshape(-1)
            zi = flat.argmax()
            zmax = flat.max().float()
            key = (zmax.clamp(min=0.0).view(torch.int32).to(torch.int64) << 32) | ((zi + g0 * m * nb) & 0xFFFFFFFF)
            st[0] = torch.maximum(st[0], key)
            st[3] += (flat < 0).sum()
        st[2] += 1
        self.counts["checked"] += 1
        self.counts["checked_flops"] += 2 * G * m * n * k

    def _grouped(self, func, args, kwargs):
        """torch._grouped_mm: one check per group, split on `offs` (cumulative group ends; one small host read
        per call). 2-D x 3-D: groups of rows of A against B[g]; 3-D x 2-D: A[g] against groups of columns of B;
        2-D x 2-D: groups of the inner dimension (one output per group); 3-D x 3-D: a bmm."""
        a, b = args[0], args[1]
        offs = kwargs.get("offs", args[2] if len(args) > 2 else None)
        bias = kwargs.get("bias", args[3] if len(args) > 3 else None)
        if bias is not None or a.dtype not in (torch.bfloat16, torch.float16) or a.shape[-1] == 0:
            raise _Skip
        out = func(*args, **kwargs)
        inj = self._take_inject()
        if inj is not None:
            _flip(out if out.dim() == 3 else out.unsqueeze(0), inj)
        rnd = ROUND[out.dtype] if out.dtype in ROUND else 0.0
        name = "aten::_grouped_mm"
        if a.dim() == 3 and b.dim() == 3:
            self._check(name, a, b, out, rnd, None)
            return out
        ends = [0] + [int(v) for v in offs.tolist()]
        for g in range(len(ends) - 1):
            lo, hi = ends[g], ends[g + 1]
            if hi <= lo:
                continue
            if a.dim() == 2 and b.dim() == 3:
                self._check(name, a[lo:hi], b[g], out[lo:hi], rnd, None)
            elif a.dim() == 3 and b.dim() == 2:
                self._check(name, a[g], b[:, lo:hi], out[:, lo:hi], rnd, None)
            else:
                self._check(name, a[:, lo:hi], b[lo:hi], out[g], rnd, None)
        return out

    # ---------------------------------------------------------------- results
    def flush(self, step: Optional[int] = None) -> list[SDCEvent]:
        rows = self.table.read(reset=True)
        new = []
        ident = None
        for r in rows:
            self.checks += r["checks"]
            self.unjudged += r["unjudged"]
            if r["z"] > self.z_alarm:
                ident = ident or device_identity(self.device)
                detail = {"op": r["name"], "z": r["z"], "row": r.get("row"), "block": r.get("block")}
                ev = SDCEvent(detector="checksum", step=step, detail=detail, identity=ident)
                self.log.add(ev)
                new.append(ev)
                if self.on_alert:
                    self.on_alert(ev)
            else:
                self.worst_clean = max(self.worst_clean, r["z"])
        self.events += new
        return new

    def coverage(self) -> dict:
        tot = self.counts["checked_flops"] + self.counts["unchecked_flops"]
        return {**self.counts, "checks": self.checks, "unjudged": self.unjudged, "alarms": len(self.events),
                "worst_clean_z": self.worst_clean, "ops_seen": len(self.slots),
                "unchecked_ops": dict(self.unchecked_ops),
                "flop_coverage": self.counts["checked_flops"] / tot if tot else 1.0}


class _Skip(Exception):
    """The op is outside what this guard checks: run it unchecked (counted)."""


def _flip(t3: torch.Tensor, inj: tuple) -> None:
    g, r, c, bit = inj
    v = t3[g, r, c:c + 1]
    if v.dtype == torch.float32:
        v.view(torch.int32).bitwise_xor_(1 << bit if bit < 31 else -(1 << 31))
    else:
        v.view(torch.int16).bitwise_xor_(1 << bit if bit < 15 else -(1 << 15))
