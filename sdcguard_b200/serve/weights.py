"""Weight scan: compares a fingerprint of every weight's bits with the one taken at registration, a budgeted
slice per poll, and optionally repairs a weight from a host copy when few of its values changed.

    scan = WeightScan(named_params, keep_host_copy=True)
    events = scan.poll(budget_mb=256)          # scans the next slice; returns SDCEvents for changed weights
    scan.full()                                # every weight now

A flipped bit in memory that holds a weight (an HBM error the ECC missed, a stray write) is silent for every
arithmetic check (the GEMM checksum rows were built from the same corrupted weight only if they are rebuilt; the
ones here are kept from registration), so the scan is the detector for it.

Reference: `WeightScan` (src/sdcguard/serve_weights.py:389), `fingerprint` (:172), repair from a host copy when
at most 64 values changed (:48-60, `_restore` :802). Here the fingerprint is `ops.fingerprint` (one batched
sm_100a kernel over all tensors of the slice).
"""
from __future__ import annotations

import time
from typing import Iterable, Optional

import torch

from ..ops.fingerprint import fingerprint
from ..utils.events import EventLog, SDCEvent, device_identity

REPAIR_MAX_VALUES = 64


class WeightScan:
    def __init__(self, named: Iterable[tuple[str, torch.Tensor]], keep_host_copy: bool = False, seed: int = 0,
                 log: Optional[EventLog] = None):
        self.names: list[str] = []
        self.tensors: list[torch.Tensor] = []
        self.left_out: list[str] = []          # named entries with nothing to fingerprint (None or empty)
        for name, t in named:
            if t is None or t.numel() == 0:
                self.left_out.append(name)
                continue
            self.names.append(name)
            self.tensors.append(t.detach())
        self.seed = seed
        self.log = log or EventLog()
        self.host = [t.cpu().clone() for t in self.tensors] if keep_host_copy else None
        self.ref = self._fp(range(len(self.tensors)))
        self.cursor = 0
        self.scanned_bytes = 0
        self.repairs = 0
        self.passes = 0                        # completed sweeps over every entry
        self.clean_at: list[Optional[float]] = [None] * len(self.tensors)   # last compare that matched
        self.changed: set = set()              # entries found changed (and not repaired back) since load

    def _fp(self, idx) -> list[tuple[int, int]]:
        idx = list(idx)
        if not idx:
            return []
        out: list = [None] * len(idx)
        by_dev: dict = {}
        for j, i in enumerate(idx):
            by_dev.setdefault(self.tensors[i].device, []).append(j)
        for dev, js in by_dev.items():
            fp = fingerprint([self.tensors[idx[j]].contiguous() for j in js], self.seed).cpu().tolist()
            for j, v in zip(js, fp):
                out[j] = tuple(v)
        return out

    def _check(self, idx: list[int], step: Optional[int]) -> list[SDCEvent]:
        now = self._fp(idx)
        t = time.time()
        events = []
        for i, fp in zip(idx, now):
            self.scanned_bytes += self.tensors[i].numel() * self.tensors[i].element_size()
            if fp == self.ref[i]:
                self.clean_at[i] = t
                continue
            detail = {"weight": self.names[i], "expected": list(self.ref[i]), "found": list(fp)}
            self.changed.add(i)
            if self.host is not None:
                detail.update(self._repair(i))
                if detail.get("repaired"):
                    self.changed.discard(i)
                    self.clean_at[i] = t
            ev = SDCEvent(detector="weights", step=step, detail=detail,
                          identity=device_identity(self.tensors[i].device))
            self.log.add(ev)
            events.append(ev)
        return events

    def _repair(self, i: int) -> dict:
        """Restores the changed values of weight i from the host copy when there are at most 64 of them."""
        t, h = self.tensors[i], self.host[i]
        cur_b = t.contiguous().cpu().view(-1).view(torch.uint8)
        ref_b = h.contiguous().view(-1).view(torch.uint8)
        changed = torch.unique(torch.nonzero(cur_b != ref_b).view(-1) // t.element_size())
        if changed.numel() > REPAIR_MAX_VALUES:
            return {"changed_values": int(changed.numel()), "repaired": False}
        with torch.no_grad():
            t.view(-1)[changed.to(t.device)] = h.view(-1)[changed].to(t.device)
        self.repairs += 1
        ok = self._fp([i])[0] == self.ref[i]
        return {"changed_values": int(changed.numel()), "repaired": ok, "positions": changed.tolist()[:16]}

    def poll(self, budget_mb: float = 256.0, step: Optional[int] = None) -> list[SDCEvent]:
        """Scan weights from the cursor until about budget_mb have been read."""
        if not self.tensors:
            return []
        budget = budget_mb * 1e6
        idx, got = [], 0
        while got < budget and len(idx) < len(self.tensors):
            i = self.cursor
            idx.append(i)
            got += self.tensors[i].numel() * self.tensors[i].element_size()
            self.cursor = (self.cursor + 1) % len(self.tensors)
            if self.cursor == 0:
                self.passes += 1
        return self._check(idx, step)

    def full(self, step: Optional[int] = None) -> list[SDCEvent]:
        ev = self._check(list(range(len(self.tensors))), step)
        self.passes += 1
        return ev

    def stats(self, now: Optional[float] = None) -> dict:
        """What the scan has verified: entries held, sweeps completed, entries never compared since load, entries
        found changed (not repaired), repairs written, and the age of the least recently verified entry (None
        while an entry has never been compared)."""
        now = time.time() if now is None else now
        never = sum(1 for c in self.clean_at if c is None)
        ok = [c for c in self.clean_at if c is not None]
        return {"entries": len(self.tensors), "passes": self.passes, "never_compared": never,
                "changed": len(self.changed), "repairs": self.repairs, "left_out": len(self.left_out),
                "oldest_age_seconds": (now - min(ok)) if ok and not never else None,
                "scanned_bytes": self.scanned_bytes}

    def digest(self) -> str:
        """One hex digest of every registered weight fingerprint (model identity)."""
        import hashlib
        h = hashlib.sha256()
        for n, fp in zip(self.names, self.ref):
            h.update(n.encode())
            h.update(str(fp).encode())
        return h.hexdigest()
