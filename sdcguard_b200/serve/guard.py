"""ServeGuard: reads the per-device check state that the serving kernels fold their results into, turns scores
above the alarm line into events, and keeps coverage counts.

State row per checked op (layout of src/sdcguard/serve.py:55-65): worst (z, location) key, worst (z, noise)
key, checks executed, checksums not judged. GEMM rows hold ABFT scores; replay rows hold 0 (identical) or inf
(a replayed row differed). `poll()` reads and clears the table once; the kernels never wait for the host.

Reference: `ServeGuard.poll` (src/sdcguard/serve.py:1090), `counts`/`coverage_report`/`worst_z` (:1030-1089).
"""
from __future__ import annotations

import math
from typing import Callable, Optional


from ..numerics import abft
from ..utils.events import EventLog, SDCEvent, device_identity


class ServeGuard:
    def __init__(self, model, z_alarm: float = abft.Z_ALARM, log: Optional[EventLog] = None,
                 on_alert: Optional[Callable[[SDCEvent], None]] = None):
        self.model = model
        self.z_alarm = z_alarm
        self.log = log or EventLog()
        self.on_alert = on_alert
        self.totals: dict[str, dict] = {}
        self.step: Optional[int] = None
        self._identity = None
        self.weight_scan = None
        self.scan_budget_mb = 0.0

    def mark_step(self, step: int) -> None:
        self.step = step

    def attach_weight_scan(self, scan, budget_mb: float = 256.0) -> None:
        """Scan `budget_mb` of weights (serve.weights.WeightScan) at every poll."""
        self.weight_scan = scan
        self.scan_budget_mb = budget_mb

    def poll(self, reset: bool = True) -> list[SDCEvent]:
        """Read every state row (one device->host copy), record events for alarms, reset the rows."""
        rows = self.model.state.read(reset=reset)
        events = []
        for r in rows:
            t = self.totals.setdefault(r["name"], {"checks": 0, "unjudged": 0, "worst_z": 0.0, "alarms": 0})
            t["checks"] += r["checks"]
            t["unjudged"] += r["unjudged"]
            z = r["z"]
            if z > t["worst_z"] or (math.isinf(z) and not math.isinf(t["worst_z"])):
                t["worst_z"] = z
            if z > self.z_alarm:
                t["alarms"] += 1
                if self._identity is None:
                    self._identity = device_identity(self.model.device)
                det = "checksum" if "GEMM" in r["name"] else "collective" if "collective" in r["name"] else "replay"
                detail = {"layer": r["name"], "z": z, "noise": r["noise"], "flat": r["flat"]}
                if "row" in r:
                    detail.update({k: r[k] for k in ("row", "block", "signed", "peer") if k in r})
                ev = SDCEvent(detector=det, step=self.step, detail=detail, identity=self._identity)
                self.log.add(ev)
                events.append(ev)
                if self.on_alert:
                    self.on_alert(ev)
        if self.weight_scan is not None:
            for ev in self.weight_scan.poll(self.scan_budget_mb, step=self.step):
                self.log.add(ev)
                events.append(ev)
                if self.on_alert:
                    self.on_alert(ev)
        return events

    def coverage_report(self) -> dict:
        checked = sum(1 for t in self.totals.values() if t["checks"] > 0)
        return {"ops": len(self.totals), "ops_checked": checked,
                "checks": sum(t["checks"] for t in self.totals.values()),
                "unjudged": sum(t["unjudged"] for t in self.totals.values()),
                "alarms": sum(t["alarms"] for t in self.totals.values()),
                "worst_clean_z": max((t["worst_z"] for t in self.totals.values() if t["alarms"] == 0), default=0.0)}

    def worst_z(self) -> float:
        return max((t["worst_z"] for t in self.totals.values()), default=0.0)
