"""Checked inference for any PyTorch model: its bf16 nn.Linear layers run on the checked tcgen05 GEMM.

    guard = attach(model)                      # or ServeGuard.attach(model, share=0.125, offset=0)
    with torch.no_grad():
        y = model(x)                           # every selected linear layer: checked GEMM, result into its state row
    events = guard.poll()                      # alarms -> SDCEvents (captured row rechecked in float64)
    guard.refresh()                            # after changing weights on purpose (a reload, a merged adapter)
    guard.verify_weights()                     # layers whose weights changed since attach (or the last refresh)
    guard.detach()                             # the original layers back

Each selected layer's class is swapped for a subclass whose forward multiplies through this package's checked GEMM
(`ops.gemm.checked_linear`): the output is the GEMM's own, and the checksum comparison runs in its epilogue, so the
layer costs one launch as before. The checksum rows are built once at attach from the weight; the GEMM reads the
live weight, so a weight that changes afterwards shows as alarms once it moves an output past the line, and
exactly in `verify_weights` (a fingerprint taken with the checksums). Calls that need gradients, or whose input is
not bf16, run the layer's original forward (unchecked, counted): this guard is for inference, the training guard
covers training.

Layers are chosen in model order with the share / offset rule of `serve.settings` (a Weyl sequence over the linear
layer index). A layer that cannot be checked is left as it is and listed with the reason: a weight that is not bf16,
not on the model's CUDA device, with n or k not a multiple of 8, or outside the share. Layers share one state table
on the device, so the serving guard's poll, coverage report, alarm capture and recheck work as for this package's
own decoder. On a CUDA device the kernels pass the first-use verification (`ops.verify`) before any layer is
swapped, and the first alarm's input row is captured on the device for the float64 recheck.

Reference: src/sdcguard/serve.py:548-1000 (`ServeGuard.attach` :619, `_make_forward` :868, `detach` :901,
`refresh` :1532, `verify_weights` :1513).
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn.functional as F

from ..ops import gemm
from ..ops.fingerprint import fingerprint
from ..train import swap
from .guard import ServeGuard
from .settings import CheckSettings, layer_selected


class AttachedModel:
    """What the serving guard reads for an attached model: one state table on the device, the checked weights by
    slot (for the float64 recheck of a captured alarm), and the layer records."""

    def __init__(self, device: torch.device, capacity: int, settings: CheckSettings):
        self.device = device
        self.state = gemm.StateTable(device, max(1, capacity))
        self.slot_weights: dict = {}
        self.settings = settings
        self.precision = "bf16"
        self.layers: list = []            # (name, module, LayerState or None, reason)
        self.fallback_calls = 0           # calls that ran the original forward (gradients, non-bf16 input)

    def check_coverage(self) -> dict:
        checked = [st for _, _, st, _ in self.layers if st is not None]
        total = sum(m.weight.numel() for _, m, _, _ in self.layers)
        return {"layers_checked": len(checked), "layers_unchecked": len(self.layers) - len(checked),
                "fp8_layers_checked": 0,
                "weights_checked_ratio": (sum(st.cw.weight.numel() for st in checked) / total) if total else 0.0}


class LayerState:
    """Stored on a swapped layer: its checked weight, state slot and load-time fingerprint."""

    def __init__(self, owner: AttachedModel, name: str, module: torch.nn.Linear, slot: int):
        self.owner, self.name, self.slot = owner, name, slot
        self.build(module)

    def build(self, module: torch.nn.Linear) -> None:
        w = module.weight.detach()
        self.cw = gemm.CheckedWeight(w, None if module.bias is None else module.bias.detach())
        self.weight_ptr = w.data_ptr()
        self.fp = fingerprint([w] + ([module.bias.detach()] if module.bias is not None else []))
        self.owner.slot_weights[self.slot] = self.cw

    def forward(self, layer: torch.nn.Linear, x: torch.Tensor) -> torch.Tensor:
        if (x.dtype != torch.bfloat16 or (torch.is_grad_enabled() and (x.requires_grad or layer.weight.requires_grad))
                or layer.weight.data_ptr() != self.weight_ptr):
            self.owner.fallback_calls += 1
            return F.linear(x, layer.weight, layer.bias)
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1])
        if x2.stride(-1) != 1:
            x2 = x2.contiguous()
        y = gemm.checked_linear(x2, self.cw, self.owner.state.state, self.slot,
                                z_alarm=self.owner.settings.z_alarm)
        return y.view(*lead, self.cw.n)


def _reason(module: torch.nn.Linear, device: torch.device) -> Optional[str]:
    w = module.weight
    if w.device.type != "cuda":
        return "not on a CUDA device"
    if w.device != device:
        return f"on {w.device}, the attached model's device is {device}"
    if w.dtype != torch.bfloat16:
        return f"weight dtype {w.dtype} (the checked GEMM multiplies bf16)"
    n, k = w.shape
    if n % 8 or k % 8:
        return f"shape {n} x {k}: n and k must be multiples of 8"
    return None


class AttachedGuard(ServeGuard):
    """The serving guard of an attached model, with attach-time operations."""

    def detach(self) -> None:
        """Give every layer its original class back; the guard keeps its totals and events."""
        for _, mod, st, _ in self.model.layers:
            if st is not None and swap.is_checked(mod):
                swap.give_back(mod)
        self.model.layers = [(n, m, None, "detached") for n, m, _, _ in self.model.layers]

    def refresh(self) -> int:
        """Rebuild the checksums and fingerprints of every checked layer from its current weights; returns how many
        layers were rebuilt. Call it after changing weights on purpose."""
        n = 0
        for _, mod, st, _ in self.model.layers:
            if st is not None:
                st.build(mod)
                n += 1
        return n

    def verify_weights(self) -> list:
        """Names of checked layers whose weight (or bias) bits differ from the fingerprint taken at attach or at the
        last refresh, or whose weight tensor was replaced."""
        out = []
        for name, mod, st, _ in self.model.layers:
            if st is None:
                continue
            ts = [mod.weight.detach()] + ([mod.bias.detach()] if mod.bias is not None else [])
            if mod.weight.data_ptr() != st.weight_ptr or not torch.equal(fingerprint(ts), st.fp):
                out.append(name)
        return out

    def layer_report(self) -> list:
        return [{"layer": n, "checked": st is not None, "reason": r} for n, _, st, r in self.model.layers]


def attach(model: torch.nn.Module, share: Optional[float] = None, offset: Optional[int] = None,
           settings: Optional[CheckSettings] = None, device=None, max_tokens: int = 0, **guard_kw) -> AttachedGuard:
    """Swap the selected bf16 nn.Linear layers of `model` for checked ones; returns their serving guard.
    max_tokens > 0: size the GEMM workspace now for every row count up to it (required before capturing the model
    in a CUDA graph)."""
    settings = settings or CheckSettings.from_env()
    if share is not None:
        settings.share = share
    if offset is not None:
        settings.offset = offset
    linears = [(n, m) for n, m in model.named_modules() if isinstance(m, torch.nn.Linear)]
    if device is None:
        cuda = [p.device for p in model.parameters() if p.device.type == "cuda"]
        device = cuda[0] if cuda else torch.device("cpu")
    device = torch.device(device)
    verification = None
    if device.type == "cuda":
        # as for this package's engine: the kernels are trusted on this device only after they reproduced their
        # references on clean and corrupted cases, and the first alarm's evidence is kept on the device
        from ..ops import verify
        verification = verify.verified(device)
        gemm.enable_capture(device)
    am = AttachedModel(device, len(linears) if device.type == "cuda" else 0, settings)
    am.verification = verification
    for i, (name, mod) in enumerate(linears):
        if swap.is_checked(mod):
            raise ValueError(f"{name} is already checked (attached twice?)")
        why = _reason(mod, device)
        if why is None and not layer_selected(i, settings.share, settings.offset):
            why = f"outside the share {settings.share:g} (offset {settings.offset})"
        if why is not None:
            am.layers.append((name, mod, None, why))
            continue
        cw_probe = mod.weight.shape
        slot = am.state.add(f"{name} (ABFT GEMM)", -(-cw_probe[0] // 128))
        st = LayerState(am, name, mod, slot)
        if max_tokens > 0:
            gemm.reserve_for_rows(device, st.cw.n, max_tokens)
        swap.take_over(mod, st)
        am.layers.append((name, mod, st, None))
    g = AttachedGuard(am, z_alarm=settings.z_alarm, **guard_kw)
    return g


def _guard_attach(cls, model, **kw):
    return attach(model, **kw)


ServeGuard.attach = classmethod(_guard_attach)
