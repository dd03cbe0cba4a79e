"""Activation-recompute check: a block run under activation checkpointing is computed twice, once in the forward
pass and again in the backward pass to rebuild its activations. On healthy hardware both runs give the same bits
(the same kernels on the same inputs), so their output fingerprints must match; a difference is a fault in one of
the two runs.

    rc = RecomputeCheck()
    y = rc.checkpoint(block, x, name="layer3")     # instead of torch.utils.checkpoint.checkpoint(block, x)
    loss.backward()
    events = rc.read(step)                          # one host read per step

Kernels that are not run-to-run deterministic (atomics in a reduction) make the check report differences on
healthy hardware; `calibrate` runs a block twice and tells whether it can be checked this way.

Reference: `RecomputeCheck` (src/sdcguard/recompute.py:148), `fingerprint` (:72), `calibrate` (:417).
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.utils.checkpoint as ckpt

from ..ops.fingerprint import fingerprint
from ..utils.events import EventLog, SDCEvent, device_identity


def _tensors(out) -> list[torch.Tensor]:
    if isinstance(out, torch.Tensor):
        return [out.detach().contiguous()]
    if isinstance(out, (tuple, list)):
        return [t.detach().contiguous() for t in out if isinstance(t, torch.Tensor)]
    return []


class RecomputeCheck:
    def __init__(self, seed: int = 0, log: Optional[EventLog] = None):
        self.seed = seed
        self.log = log or EventLog()
        self.pairs: list[tuple[str, torch.Tensor, torch.Tensor]] = []
        self._first: dict[int, tuple[str, torch.Tensor]] = {}
        self._n = 0
        self.checks = 0

    def checkpoint(self, fn: Callable, *args, name: Optional[str] = None, **kw):
        key = self._n
        self._n += 1
        label = name or getattr(fn, "__name__", type(fn).__name__)

        def run(*a):
            out = fn(*a, **kw)
            fp = fingerprint(_tensors(out), self.seed)
            if key not in self._first:
                self._first[key] = (label, fp)
            else:
                lab, first = self._first.pop(key)
                self.pairs.append((lab, first, fp))
            return out

        # the recompute must run to the end of the block (its outputs are fingerprinted), not stop early
        with ckpt.set_checkpoint_early_stop(False):
            return ckpt.checkpoint(run, *args, use_reentrant=False)

    def read(self, step: Optional[int] = None) -> list[SDCEvent]:
        """Compares every forward / recompute pair recorded since the last read (one device->host copy)."""
        events = []
        pairs, self.pairs = self.pairs, []
        self._first.clear()
        self._n = 0
        if not pairs:
            return events
        same = [torch.equal(a, b) for _, a, b in pairs]
        self.checks += len(pairs)
        for (lab, a, b), ok in zip(pairs, same):
            if not ok:
                ev = SDCEvent(detector="recompute", step=step,
                              detail={"block": lab, "forward": a.cpu().tolist(), "recompute": b.cpu().tolist()},
                              identity=device_identity(a.device))
                self.log.add(ev)
                events.append(ev)
        return events


def calibrate(fn: Callable, *args, runs: int = 2, seed: int = 0) -> bool:
    """True when `fn(*args)` gives bit-identical outputs on repeated runs (the block can be checked)."""
    with torch.no_grad():
        fps = [fingerprint(_tensors(fn(*args)), seed).cpu() for _ in range(runs)]
    return all(torch.equal(fps[0], f) for f in fps[1:])
