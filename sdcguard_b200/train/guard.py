"""Training guard: every protected nn.Linear runs its forward GEMM and both backward GEMMs (dX = dY W and
dW = dY^T X) through the checked sm_100a GEMM, so all three carry the ABFT check of their fp32 accumulators.
Results fold into a device state table; the host reads it once per checked step.

    guard = SDCGuard(check_every=10)
    guard.protect(model)                        # every nn.Linear's forward goes through the guard (class swap)
    for step, batch in enumerate(loader):
        with guard.at_step(step):               # checked on steps where step % check_every == 0
            loss = model(batch).loss
            loss.backward()
        opt.step(); opt.zero_grad()
    guard.events                                # SDCEvents (detector "checksum", detail: layer, phase, row, block)

The backward operands are laid out for the kernel's C = A B^T form: dX = dY (W^T)^T with W^T materialised, and
dW = (dY^T) (X^T)^T with dY^T and X^T materialised. W^T and X^T come with their checksum rows from one device pass
over W and X (`CheckedWeight.of_transpose`, `csrc/train_prep.cu`), and the forward weight's checksum rows after an
optimizer step from one pass over W (`CheckedWeight.on_device`): no fp64 PyTorch reductions on the training path.
Shapes the kernel does not take (dimensions not multiples of 8) run unchecked and are counted in `coverage()`.

Reference: `SDCGuard` (src/sdcguard/guard.py:788): `protect` :1096 swaps nn.Linear for a checked-linear autograd
function covering fwd, dX and dW (`_CheckedLinear` :448, `_checked_forward` :471, `_checked_backward` :497), checks
queued and read back once per step (`_queue` :1739, `_flush` :1882), `at_step` :1420 with an every-N schedule.
"""
from __future__ import annotations

import contextlib
from typing import Optional

import torch
import torch.nn.functional as F

from ..numerics import abft
from ..ops import gemm
from ..utils.events import EventLog, SDCEvent, device_identity

PHASES = ("fwd", "dx", "dw")


class SDCError(RuntimeError):
    """Raised at the read-back of a checked step when the guard was built with raise_on_alert=True and a check
    found corruption; .events holds the step's alerts."""

    def __init__(self, message: str, events: Optional[list] = None):
        super().__init__(message)
        self.events = events or []


class _Cache:
    """Checksum data of one weight, built once per checked step (and again if the weight changes within the step):
    the optimizer changes weights between steps, and fused optimizers (AdamW(fused=True)) do so without bumping the
    tensors' version counters, so a version check alone would keep stale checksums and a stale bf16 copy. A weight
    kept in fp32 (mixed precision under autocast) is checked as its bf16 copy, which is what autocast would feed the
    GEMM. A bf16 weight and an fp32 bias are used in place: nothing changes them between the forward and the backward
    of a checked step, and the host reads the step's checks (and replays alarms) before the optimizer runs."""

    def __init__(self, guard: "SDCGuard"):
        self.guard = guard
        self.key = None
        self.cw: Optional[gemm.CheckedWeight] = None
        self.cwT: Optional[gemm.CheckedWeight] = None

    def get(self, w: torch.Tensor, b: Optional[torch.Tensor]):
        key = (self.guard.epoch, w.data_ptr(), w._version, None if b is None else (b.data_ptr(), b._version))
        if key != self.key:
            wb = w.detach().to(torch.bfloat16)
            bb = None if b is None else b.detach()
            self.cw = gemm.CheckedWeight.on_device(wb, bb)
            self.cwT = None
            self.key = key
        return self.cw

    def get_t(self):
        if self.cwT is None:
            self.cwT = gemm.CheckedWeight.of_transpose(self.cw.weight)
        return self.cwT


def _fwd_gemm(mod: "CheckedLinear", x, w, b):
    """The checked forward GEMM of a protected layer: x (..., k) bf16 -> (..., n) bf16, with the bf16 weight used
    (a copy of an fp32 weight, made once per version)."""
    g = mod.guard
    k = x.shape[-1]
    x2 = x.reshape(-1, k).contiguous()
    cw = mod.cache.get(w, b)
    g._keep(mod.slots["fwd"], cw)
    y = gemm.checked_linear(x2, cw, g.table.state, mod.slots["fwd"], z_alarm=g.z_alarm,
                            inject=g._take_inject(mod.name, "fwd"))
    return y.view(*x.shape[:-1], w.shape[0]), x2, cw.weight


def _bwd_gemms(mod: "CheckedLinear", dy, x2, wb, xshape, need_x: bool, need_w: bool, need_b: bool):
    """dX = dY W and dW = dY^T X on the checked GEMM (dW unchecked when the token count is not a multiple of 8),
    db = the column sums of dY in fp32. wb: the bf16 weight of the forward."""
    g = mod.guard
    n = wb.shape[0]
    dy2 = dy.reshape(-1, n).to(torch.bfloat16).contiguous()
    m = dy2.shape[0]
    dx = dw = db = None
    if need_x:
        g._keep(mod.slots["dx"], mod.cache.get_t())
        dx = gemm.checked_linear(dy2, mod.cache.get_t(), g.table.state, mod.slots["dx"], z_alarm=g.z_alarm,
                                 inject=g._take_inject(mod.name, "dx")).view(xshape)
    if need_w:
        if m % 8 == 0:
            xt = gemm.CheckedWeight.of_transpose(x2)            # X^T (k, m): rows = output columns of dW
            g._keep(mod.slots["dw"], xt)
            dw = gemm.checked_linear(gemm.transpose(dy2), xt, g.table.state, mod.slots["dw"],
                                     z_alarm=g.z_alarm, inject=g._take_inject(mod.name, "dw"))
        else:
            dw = dy2.t() @ x2
            g.unchecked += 1
    if need_b:
        db = dy2.sum(0, dtype=torch.float32)
    return dx, dw, db


class _CheckedLinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, mod):
        y, x2, wb = _fwd_gemm(mod, x, w, b)
        ctx.save_for_backward(x2, wb)
        ctx.wdtype = w.dtype
        ctx.mod = mod
        ctx.has_bias = b is not None
        ctx.bdtype = None if b is None else b.dtype
        ctx.xshape = x.shape
        return y

    @staticmethod
    def backward(ctx, dy):
        x2, wb = ctx.saved_tensors
        need_b = ctx.has_bias and ctx.needs_input_grad[2]
        dx, dw, db = _bwd_gemms(ctx.mod, dy, x2, wb, ctx.xshape, ctx.needs_input_grad[0], ctx.needs_input_grad[1],
                                need_b)
        return (dx, None if dw is None else dw.to(ctx.wdtype), None if db is None else db.to(ctx.bdtype), None)


class CheckedLinear:
    """The guard's state of one protected linear layer: its name, check slots and checksum cache. The layer object
    itself stays in the model (train.swap gives it a subclass whose forward calls `forward` here), so copies,
    pickles and references to the layer behave as they did."""

    def __init__(self, lin: torch.nn.Linear, guard: "SDCGuard", name: str):
        self.layer = lin
        self.in_features, self.out_features = lin.in_features, lin.out_features
        self.guard = guard
        self.name = name
        self.cache = _Cache(guard)
        self.slots = {}
        n, k = lin.out_features, lin.in_features
        nbs = {"fwd": -(-n // abft.BLOCK), "dx": -(-k // abft.BLOCK), "dw": -(-k // abft.BLOCK)}
        for ph in PHASES:
            self.slots[ph] = guard.table.add(f"{name}.{ph} (ABFT GEMM)", nbs[ph])
        from . import compiled
        self.state_id = compiled.register(self)      # (at protect time: the traced forward only reads it)

    @property
    def weight(self):
        return self.layer.weight

    # ---- the operators of train.compiled call these (under torch.compile, and on DTensor local shards)
    def runnable(self, x, w) -> bool:
        ok = (self.guard.active and x.is_cuda and x.shape[-1] % 8 == 0 and w.shape[0] % 8 == 0 and
              x.dtype in (torch.bfloat16, torch.float32) and w.dtype in (torch.bfloat16, torch.float32))
        if self.guard.active and not ok:
            self.guard.unchecked += 1
        return ok

    def checked_forward(self, x, w, b):
        self.guard.checked_calls += 1
        y, _, _ = _fwd_gemm(self, x.to(torch.bfloat16), w, b)
        return y.to(x.dtype)

    def checked_backward(self, gy, x, w, need_x, need_w, need_b):
        c = self.cache
        if c.cw is None or c.key[:3] != (self.guard.epoch, w.data_ptr(), w._version):
            c.get(w, None)                       # the forward's cache entry is normally still current
        xb = x.to(torch.bfloat16)
        dx, dw, db = _bwd_gemms(self, gy, xb.reshape(-1, x.shape[-1]).contiguous(), self.cache.cw.weight, x.shape,
                                need_x, need_w, need_b)
        return (None if dx is None else dx.to(x.dtype), None if dw is None else dw.to(w.dtype),
                None if db is None else db.to(w.dtype))

    def forward(self, layer: torch.nn.Linear, x):
        g = self.guard
        w, b = layer.weight, layer.bias
        # bf16 operands, or fp32 ones under a bf16 autocast region (checked as the bf16 copies autocast would use)
        amp = x.is_cuda and torch.is_autocast_enabled("cuda") and torch.get_autocast_dtype("cuda") == torch.bfloat16
        ok = (g.active and x.is_cuda and self.in_features % 8 == 0 and self.out_features % 8 == 0 and
              ((x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16) or
               (amp and x.dtype in (torch.float32, torch.bfloat16) and w.dtype == torch.float32)))
        if not ok:
            if g.active:
                g.unchecked += 1
            return F.linear(x, w, b)
        if torch.compiler.is_compiling():
            from . import compiled
            return compiled.checked_linear(x, w, b, self.state_id)
        g.checked_calls += 1
        xb = x if x.dtype == torch.bfloat16 else x.to(torch.bfloat16)
        with torch.autocast("cuda", enabled=False):
            return _CheckedLinearFn.apply(xb, w, b, self)


class SDCGuard:
    def __init__(self, check_every: int = 1, z_alarm: float = abft.Z_ALARM, device=None,
                 log: Optional[EventLog] = None, on_alert=None, replicas: bool = False, replica_group=None,
                 recompute: bool = False, exact_reductions: bool = True, keep_evidence: bool = True,
                 evidence_dir: Optional[str] = None, confirm_runs: int = 20, raise_on_alert: bool = False):
        """replicas: after each checked step every rank shares (a multiple of check_every, an after_restart()
        window), compare the protected model's weight fingerprints across the data-parallel ranks (a collective).
        recompute: blocks run through guard.checkpoint() are fingerprinted in the forward and in the backward
        recompute on checked steps. exact_reductions: on checked steps, PyTorch's bf16 GEMMs (the unchecked ones,
        attention's among them) keep their split-K partial sums in fp32. keep_evidence: the operands of each
        checked GEMM of a step are kept until the step's check is read, so an alarm comes with its input row,
        a float64 recheck and `confirm_runs` replays of the flagged block on this GPU; evidence_dir: each such
        alarm is also saved there (torch.save, loadable with weights_only=True). raise_on_alert: the read-back of
        a checked step that found corruption raises SDCError (after logging and evidence)."""
        self.check_every = max(1, int(check_every))
        self.raise_on_alert = raise_on_alert
        self.epoch = 0                      # checked steps begun: the checksum caches are per checked step
        self.replicas, self.replica_group = replicas, replica_group
        self.exact_reductions = exact_reductions
        self.keep_evidence, self.evidence_dir, self.confirm_runs = keep_evidence, evidence_dir, confirm_runs
        self._kept: dict = {}
        self._model_ref = None
        self.recompute = None
        if recompute:
            from .recompute import RecomputeCheck
            self.recompute = RecomputeCheck()
        self.z_alarm = z_alarm
        self.device = torch.device(device or "cuda")
        self.table = gemm.StateTable(self.device, 512)
        self.log = log or EventLog()
        self.on_alert = on_alert
        self.events: list[SDCEvent] = []
        self.active = False
        self.step: Optional[int] = None
        self.checked_calls = 0
        self.unchecked = 0
        self.checks = 0
        self.steps_checked = 0
        self.worst_clean = 0.0
        self._inject: dict = {}
        self.modules: list[CheckedLinear] = []

    def protect(self, model: torch.nn.Module) -> torch.nn.Module:
        if self.device.type == "cuda":
            from ..ops import verify
            self.verification = verify.verified(self.device)   # the kernels reproduced their references here
        from . import swap
        import weakref
        self._model_ref = weakref.ref(model)
        if self.device.type == "cuda" and self.keep_evidence:
            gemm.enable_capture(self.device)
        for name, mod in list(model.named_modules()):
            if isinstance(mod, torch.nn.Linear) and not swap.is_checked(mod):
                st = CheckedLinear(mod, self, name)
                swap.take_over(mod, st)
                self.modules.append(st)
        return model

    def release(self, model: torch.nn.Module) -> torch.nn.Module:
        """Undo protect(): every layer this guard took over gets its original class back."""
        from . import swap
        mine = {id(st) for st in self.modules}
        for _, mod in model.named_modules():
            st = swap.state_of(mod)
            if st is not None and id(st) in mine:
                swap.give_back(mod)
        return model

    def should_check(self, step: int) -> bool:
        """True on every `check_every`-th step, and on every step of a window opened by after_restart() or observe()."""
        if step % self.check_every == 0:
            return True
        windows = [w for w in (getattr(self, "_dense", None), getattr(self, "_spike", None)) if w is not None]
        return any(a <= step < b for a, b in windows)

    def after_restart(self, step: int, steps: int = 50) -> "SDCGuard":
        """Call when training resumes from a checkpoint (after a crash, say): every step from `step` to
        `step + steps` is checked, so a GPU that is still bad is named before it costs another run."""
        self._dense = (step, step + steps)
        return self

    def observe(self, step: int, loss=None, grad_norm=None, steps: int = 50, threshold: float = 8.0) -> bool:
        """Watch the loss and gradient norm (numbers, after each step). When one is not finite, or lies more than
        `threshold` robust deviations (1.4826 x median absolute deviation) above the median of its last 200 values
        (once 20 are known), every step from the next one for `steps` steps is checked. A loss or gradient spike is
        often the first sign of corruption; this turns it into a checked window. Returns True when it opened or
        extended one; the reasons go to `self.anomalies`."""
        import collections
        import math
        import statistics
        hist = getattr(self, "_watch", None)
        if hist is None:
            hist = self._watch = {}
            self.anomalies = []
        why = []
        for name, v in (("loss", loss), ("grad_norm", grad_norm)):
            if v is None:
                continue
            try:
                v = float(v)
            except (TypeError, ValueError):
                continue
            h = hist.setdefault(name, collections.deque(maxlen=200))
            if not math.isfinite(v):
                why.append(f"{name} is {v}")
                continue
            if len(h) >= 20:
                med = statistics.median(h)
                spread = max(statistics.median(abs(x - med) for x in h) * 1.4826, 1e-3 * abs(med), 1e-12)
                if (v - med) / spread > threshold:
                    why.append(f"{name} {v:.4g}, recent median {med:.4g}")
            h.append(v)
        if not why:
            return False
        start = step + 1
        prev = getattr(self, "_spike", None)
        end = max(prev[1] if prev is not None and prev[1] > start else 0, start + steps)
        self._spike = (start, end)
        self.anomalies.append({"step": step, "why": why, "checked_through": end - 1})
        return True

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
        self.step = step
        self.active = force or step % self.check_every == 0
        if self.active:
            self.epoch += 1
        flag = torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction
        if self.active and self.exact_reductions:
            torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = False
        try:
            yield self
        finally:
            torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = flag
            if self.active:
                self.flush(step)
                if self.replicas and (step % self.check_every == 0 or self._in_window(step, "_dense")):
                    self._replica_check(step)
            self.active = False
            self._kept.clear()

    def _in_window(self, step: int, name: str) -> bool:
        w = getattr(self, name, None)
        return w is not None and w[0] <= step < w[1]

    def _replica_check(self, step: int) -> None:
        """Weight fingerprints voted across the data-parallel ranks (only on steps every rank checks: a rank that
        entered the collective alone would wait for the others)."""
        import torch.distributed as dist
        model = self._model_ref() if self._model_ref is not None else None
        if model is None or not (dist.is_available() and dist.is_initialized()):
            return
        if dist.get_world_size(self.replica_group) < 2:
            return
        from .replica import check_replicas
        for ev in check_replicas(list(model.parameters()), group=self.replica_group, step=step):
            self._emit(ev)

    def checkpoint(self, fn, *args, name: Optional[str] = None, **kw):
        """Activation checkpointing of a block (torch.utils.checkpoint, non-reentrant); on checked steps with
        recompute=True the block's forward and its backward recompute are fingerprinted and compared."""
        import torch.utils.checkpoint as ckpt
        if self.active and self.recompute is not None:
            return self.recompute.checkpoint(fn, *args, name=name, **kw)
        return ckpt.checkpoint(fn, *args, use_reentrant=False, **kw)

    def _keep(self, slot: int, cw) -> None:
        if self.keep_evidence and self.active:
            self._kept[slot] = cw

    def _emit(self, ev: SDCEvent) -> None:
        self.log.add(ev)
        self.events.append(ev)
        if self.on_alert:
            self.on_alert(ev)

    def inject_next(self, layer: str, phase: str, row: int, col: int, bit: int) -> None:
        """Fault injection: flip `bit` of fp32 accumulator (row, col) of the next `phase` GEMM of `layer`."""
        self._inject[(layer, phase)] = (row, col, 1 << bit)

    def _take_inject(self, layer: str, phase: str):
        return self._inject.pop((layer, phase), None)

    def flush(self, step: Optional[int] = None) -> list[SDCEvent]:
        from ..utils.trace import nvtx_range
        with nvtx_range("sdcguard.flush"):
            return self._flush(step)

    def _flush(self, step: Optional[int] = None) -> list[SDCEvent]:
        rows = self.table.read(reset=True)
        if self.recompute is not None:
            for ev in self.recompute.read(step):
                self._emit(ev)
        self.steps_checked += 1
        new = []
        ident = None
        for r in rows:
            self.checks += r["checks"]
            if r["z"] > self.z_alarm:
                ident = ident or device_identity(self.device)
                layer, ph = r["name"].split(" ")[0].rsplit(".", 1)
                ev = SDCEvent(detector="checksum", step=step,
                              detail={"layer": layer, "phase": ph, "z": r["z"], "row": r.get("row"),
                                      "block": r.get("block"), "noise": r["noise"]}, identity=ident)
                self.log.add(ev)
                new.append(ev)
                if self.on_alert:
                    self.on_alert(ev)
            else:
                self.worst_clean = max(self.worst_clean, r["z"])
        self.events += new
        if new and self.device.type == "cuda" and self.keep_evidence:
            self._evidence(new, step)
        if new and self.raise_on_alert:
            where = ", ".join(sorted({str(e.detail.get("layer", e.detector)) for e in new})[:4])
            raise SDCError(f"sdcguard: {len(new)} alert(s) at step {step}: {where}", new)
        return new

    def _evidence(self, new: list, step) -> None:
        """The device's captured alarm (input row and block sums, recorded by the GEMM that alarmed): a float64
        recheck against that GEMM's B operand kept for the step, `confirm_runs` replays of the block on this GPU,
        and an evidence file when evidence_dir is set."""
        cap = gemm.read_capture(self.device)
        if cap is None:
            return
        slot = self.table.slot_of(cap["state_row"])
        if slot is None:
            return
        name = self.table.names[slot]
        layer, ph = name.split(" ")[0].rsplit(".", 1)
        cw = self._kept.get(slot)
        rec = gemm.recheck_capture(cap, cw) if cw is not None and cw.k == cap["k"] else None
        confirm = self._confirm(cap, cw) if cw is not None and cw.k == cap["k"] else None
        kept = {k: v for k, v in cap.items() if k != "x_row"}
        for ev in new:
            if ev.detail.get("layer") == layer and ev.detail.get("phase") == ph:
                ev.detail.update(captured=kept, recheck=rec, confirm=confirm)
                break
        if self.evidence_dir and cw is not None:
            import os
            os.makedirs(self.evidence_dir, exist_ok=True)
            b = cap["block"]
            path = os.path.join(self.evidence_dir, f"step{step}_{layer}_{ph}_r{cap['row']}_b{b}.pt")
            torch.save({"format": "sdcguard-b200-train-evidence/1", "layer": layer, "phase": ph, "step": step,
                        "x_row": cap["x_row"], "w_block": cw.weight[b * abft.BLOCK:(b + 1) * abft.BLOCK].cpu(),
                        "captured": kept, "recheck": rec, "confirm": confirm}, path)
            for ev in new:
                if ev.detail.get("layer") == layer and ev.detail.get("phase") == ph:
                    ev.detail["evidence"] = path

    def _confirm(self, cap: dict, cw) -> dict:
        """Replays of the flagged (row, block) on this GPU with the checked GEMM: how many of `confirm_runs` alarm
        or leave the float64 envelope (a fault that follows the device and its kernel reproduces; a transient
        one does not)."""
        b = cap["block"]
        c0, c1 = b * abft.BLOCK, min((b + 1) * abft.BLOCK, cw.n)
        x = cap["x_row"].to(self.device).view(1, -1).contiguous()
        wb = cw.weight[c0:c1].contiguous()
        cwb = gemm.CheckedWeight(wb)
        tab = gemm.StateTable(self.device, 1)
        s = tab.add("confirm", cwb.nb)
        ref = (wb.double() @ x.double().view(-1))
        env = 2.0 ** -8 * ref.abs() + 1.01 * x.shape[1] * 2.0 ** -24 * (wb.double().abs() @ x.double().abs().view(-1))
        wrong = alarms = 0
        for _ in range(max(0, self.confirm_runs)):
            y = gemm.checked_linear(x, cwb, tab.state, s)[0].double()
            wrong += int(((y - ref).abs() > env + 1e-30).any())
            alarms += int(tab.read(reset=True)[0]["z"] > self.z_alarm)
        return {"runs": self.confirm_runs, "wrong_outputs": wrong, "alarms": alarms,
                "reproduced": wrong + alarms > 0}

    def coverage(self) -> dict:
        return {"layers": len(self.modules), "checked_calls": self.checked_calls, "unchecked_calls": self.unchecked,
                "checks": self.checks, "steps_checked": self.steps_checked, "alarms": len(self.events),
                "worst_clean_z": self.worst_clean}
