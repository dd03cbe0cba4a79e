"""ABFT check of fp32 linear layers on the CPU (the CPU configuration of the benchmark: GPT-2 small in fp32,
every nn.Linear checked). The reference checks bf16/fp16 matmuls only and returns no check for fp32
(src/sdcguard/checksum.py:423-425, serve.py:670-675); this module extends the same block-checksum idea to fp32.

For y = x W^T + b (fp32 GEMM, here MKL through torch), each 128-column block b of each output row gets two sums,
plain and with fixed +-1 signs (the signs of `abft.sign_mask`), compared in float64 against the expected side
x . (block sums of W) + block sums of b, computed once per weight. Noise model of the fp32 accumulation: for a
dot product of length K the rounding error of each output is about u sqrt(K) ||x_k w_jk||_2 (u = 2^-24), so the
error of a block sum has standard deviation

    sigma_b = u * (sqrt(K) * sqrt(sum_j sum_k x_k^2 w_jk^2) + sqrt(128) * ||y_b||_2)

(the second term is the final rounding of every output), with sum_j w_jk^2 per block precomputed. The score is
max(|plain - expected|, |signed - expected_signed|) / sigma_b; an alarm is a score above 6. A non-finite output
with finite inputs is an alarm (infinite score).
"""
from __future__ import annotations

import math
from typing import Callable, Optional

import torch
import torch.nn.functional as F
from torch.utils._python_dispatch import _disable_current_modes

from . import abft

U32 = 2.0 ** -24


class CPUCheckState:
    """Worst score per named layer, counts, and the alarms with their location."""

    def __init__(self):
        self.worst: dict[str, float] = {}
        self.checks = 0
        self.alarms: list[dict] = []
        self.calls = 0
        self.call_z: list[float] = []            # worst score of every call, in call order
        self.probes: dict[int, dict] = {}        # call -> record to receive the noise scale at (row, block)
        self.unjudged = 0                        # checksums whose inputs were non-finite

    def record(self, name: str, call: int, z: torch.Tensor, z_alarm: float, sigma: torch.Tensor) -> None:
        self.checks += z.numel()
        zmax = float(z.max()) if z.numel() else 0.0
        self.call_z.append(zmax)
        self.worst[name] = max(self.worst.get(name, 0.0), zmax)
        pr = self.probes.pop(call, None)
        if pr is not None:
            pr["sigma"] = float(sigma[pr["row"], pr["block"]])
        if zmax > z_alarm:
            flat = int(torch.argmax(z))
            row, block = divmod(flat, z.shape[1])
            self.alarms.append({"layer": name, "call": call, "row": row, "block": block, "z": zmax})


class CheckedLinearCPU(torch.nn.Module):
    """An nn.Linear (fp32) whose every output block is checked. `inject` (optional) corrupts the GEMM output
    before the check, as a fault in the GEMM would."""

    def __init__(self, lin: torch.nn.Linear, name: str, state: CPUCheckState, z_alarm: float = abft.Z_ALARM,
                 inject: Optional[Callable] = None):
        super().__init__()
        self.lin = lin
        self.name = name
        self.state = state
        self.z_alarm = z_alarm
        self.inject = inject
        self.refresh()

    @torch.no_grad()
    def refresh(self) -> None:
        """Rebuild the weight block sums (after the weights change, e.g. an optimizer step)."""
        W = self.lin.weight.detach().double()
        n, k = W.shape
        nb = -(-n // abft.BLOCK)
        Wp = torch.zeros(nb * abft.BLOCK, k, dtype=torch.float64)
        Wp[:n] = W
        Wp = Wp.view(nb, abft.BLOCK, k)
        s = abft.sign_vector(abft.sign_mask()).view(1, abft.BLOCK, 1)
        self.nb, self.k, self.n = nb, k, n
        self.wsum = Wp.sum(1).t().contiguous()                  # (k, nb)
        self.wsgn = (Wp * s).sum(1).t().contiguous()
        self.w2 = (Wp * Wp).sum(1).t().contiguous()             # (k, nb)
        self.signs = s.view(1, 1, abft.BLOCK)
        if self.lin.bias is not None:
            b = torch.zeros(nb * abft.BLOCK, dtype=torch.float64)
            b[:n] = self.lin.bias.detach().double()
            b = b.view(nb, abft.BLOCK)
            self.bsum, self.bsgn = b.sum(1), (b * s.view(1, abft.BLOCK)).sum(1)
        else:
            self.bsum = self.bsgn = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = F.linear(x, self.lin.weight, self.lin.bias)
        call = self.state.calls
        self.state.calls += 1
        if self.inject is not None:
            self.inject(y, self.name, call)
        with torch.no_grad(), _disable_current_modes():
            z, sig = self.scores(x, y)
            self.state.record(self.name, call, z, self.z_alarm, sig)
        return y

    @torch.no_grad()
    def scores(self, x: torch.Tensor, y: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """(m, nb) scores and noise scales of the output blocks."""
        X = x.reshape(-1, self.k).double()
        m = X.shape[0]
        y2 = y.detach().reshape(m, self.n)
        if self.n % abft.BLOCK:
            yp = torch.zeros(m, self.nb * abft.BLOCK, dtype=y2.dtype)
            yp[:, : self.n] = y2
            y2 = yp
        Y = y2.view(m, self.nb, abft.BLOCK)
        s32 = self.signs.to(Y.dtype)
        act = Y.sum(-1, dtype=torch.float64)
        acts = (Y * s32).sum(-1, dtype=torch.float64)          # exact: sign changes only
        ysq = torch.linalg.vector_norm(Y, dim=-1, dtype=torch.float64).pow(2)     # no fp32 overflow
        exp, exps = X @ self.wsum, X @ self.wsgn
        if self.bsum is not None:
            exp, exps = exp + self.bsum, exps + self.bsgn
        sig = U32 * (math.sqrt(self.k) * ((X * X) @ self.w2).sqrt() + math.sqrt(abft.BLOCK) * ysq.sqrt())
        sig = sig + abft.ABS_FLOOR
        z = torch.maximum((act - exp).abs(), (acts - exps).abs()) / sig
        xfin = torch.isfinite(X).all(-1, keepdim=True)                      # rows with finite inputs
        bad = (~torch.isfinite(act) | ~torch.isfinite(acts)) & xfin
        z = torch.where(bad, torch.full_like(z, math.inf), z)
        # rows whose inputs are already non-finite (a fault upstream) cannot be judged here
        self.state.unjudged += int((~xfin).sum()) * self.nb
        z = torch.where(xfin, z, torch.zeros_like(z))
        return z, sig


def protect_cpu(model: torch.nn.Module, state: Optional[CPUCheckState] = None, inject: Optional[Callable] = None,
                z_alarm: float = abft.Z_ALARM) -> CPUCheckState:
    """Replaces every nn.Linear of the model by a CheckedLinearCPU (in place). Returns the shared state."""
    state = state or CPUCheckState()
    for parent_name, parent in list(model.named_modules()):
        for child_name, child in list(parent.named_children()):
            if isinstance(child, torch.nn.Linear):
                full = f"{parent_name}.{child_name}" if parent_name else child_name
                setattr(parent, child_name, CheckedLinearCPU(child, full, state, z_alarm, inject))
    return state
