"""Data-parallel canary: every rank runs the same batch through the model; a forward hook fingerprints every leaf
module's output; the ranks exchange the fingerprints and vote per module call. A rank whose output differs from
the majority is the suspect (its GPU computed something else from the same inputs and weights).

    canary = Canary(model)           # hooks on every leaf module
    with canary.recording():
        model(same_batch_on_every_rank)
    events = canary.check(step)      # collective: identical result on every rank

Reference: `Canary` (src/sdcguard/canary.py:53-154: hook fingerprints, all_gather, majority vote per layer
call). The fingerprints here are the two-sum bit fingerprint of `ops.fingerprint` plus dtype and shape codes.
"""
from __future__ import annotations

import contextlib
from collections import Counter
from typing import Optional

import torch
import torch.distributed as dist

from ..ops.fingerprint import fingerprint
from ..utils.events import EventLog, SDCEvent, device_identity, gather_identities, job_rank, suspect_event

_DTYPES = {d: i for i, d in enumerate([torch.float32, torch.float16, torch.bfloat16, torch.float64, torch.int64,
                                        torch.int32, torch.uint8, torch.bool, torch.int8, torch.int16])}


def _shape_code(t: torch.Tensor) -> int:
    h = 1469598103934665603
    for d in t.shape:
        h = ((h ^ int(d)) * 1099511628211) & ((1 << 63) - 1)
    return h


def majority(rows: list[tuple]) -> tuple[Optional[tuple], list[int]]:
    """Most common row and the indices (ranks) that differ from it; no majority (tie) -> (None, all)."""
    c = Counter(rows)
    (top, n), *rest = c.most_common()
    if rest and rest[0][1] == n:
        return None, list(range(len(rows)))
    return top, [i for i, r in enumerate(rows) if r != top]


class Canary:
    def __init__(self, model: torch.nn.Module, group=None, seed: int = 0, log: Optional[EventLog] = None):
        self.group = group
        self.seed = seed
        self.log = log or EventLog()
        self.calls: list[tuple[str, torch.Tensor]] = []
        self._on = False
        self._hooks = []
        for name, m in model.named_modules():
            if next(m.children(), None) is None:
                self._hooks.append(m.register_forward_hook(self._hook(name or type(m).__name__)))

    def _hook(self, name):
        def fn(mod, inp, out):
            if not self._on:
                return
            t = out[0] if isinstance(out, (tuple, list)) else out
            if isinstance(t, torch.Tensor):
                self.calls.append((name, t.detach().contiguous()))
        return fn

    @contextlib.contextmanager
    def recording(self):
        self.calls = []
        self._on = True
        try:
            yield self
        finally:
            self._on = False

    def remove(self) -> None:
        for h in self._hooks:
            h.remove()

    def fingerprints(self) -> torch.Tensor:
        """(calls, 4) int64: two-sum fingerprint, dtype code, shape code of each recorded output."""
        if not self.calls:
            return torch.zeros(0, 4, dtype=torch.int64)
        fp = fingerprint([t for _, t in self.calls], self.seed).cpu()
        meta = torch.tensor([[_DTYPES.get(t.dtype, 99), _shape_code(t)] for _, t in self.calls], dtype=torch.int64)
        return torch.cat([fp, meta], dim=1)

    def check(self, step: Optional[int] = None) -> list[SDCEvent]:
        """Collective. Votes per module call; returns one event per call with a dissenting rank (same list on
        every rank). A rank that recorded a different number of calls is a suspect too."""
        mine = self.fingerprints()
        world = dist.get_world_size(self.group) if dist.is_initialized() else 1
        counts = [None] * world
        if world > 1:
            dist.all_gather_object(counts, mine.shape[0], group=self.group)
        else:
            counts = [mine.shape[0]]
        n = max(counts)
        pad = torch.full((n, 4), -1, dtype=torch.int64)
        pad[: mine.shape[0]] = mine
        backend_dev = self._comm_device()
        gathered = [torch.empty(n, 4, dtype=torch.int64, device=backend_dev) for _ in range(world)]
        if world > 1:
            dist.all_gather(gathered, pad.to(backend_dev), group=self.group)
        else:
            gathered = [pad]
        g = torch.stack([x.cpu() for x in gathered])          # (world, n, 4)
        events = []
        names = [nm for nm, _ in self.calls] + ["?"] * (n - len(self.calls))
        votes = [majority([tuple(g[r, c].tolist()) for r in range(world)]) for c in range(n)]
        if not any(bad for _, bad in votes):
            return events
        # every rank saw the same votes: they exchange identities together, once, to name the suspects' GPUs
        dev = self.calls[0][1].device if self.calls else None
        ids = gather_identities(self.group, dev) if world > 1 else [device_identity(dev)]
        me = dist.get_rank(self.group) if world > 1 else 0
        for c, (top, bad) in enumerate(votes):
            if bad:
                ev = suspect_event("canary", step, bad, ids, me,
                                   {"call": c, "module": names[c], "no_majority": top is None},
                                   to_job_rank=lambda r: job_rank(self.group, r))
                self.log.add(ev)
                events.append(ev)
        return events

    def _comm_device(self):
        if dist.is_initialized() and dist.get_backend(self.group) == "nccl":
            return torch.device("cuda", torch.cuda.current_device())
        return torch.device("cpu")
