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

import torch


from ..numerics import abft
from ..utils.events import EventLog, SDCEvent, device_identity
from ..utils.trace import nvtx_range


CONFIRMING_RECHECKS = ("output_wrong", "both_wrong", "weights_changed")


def confirmed(ev: SDCEvent) -> bool:
    """Does an event carry its own evidence of a wrong result? A captured GEMM alarm whose float64 recheck shows a
    wrong output or changed weights, or a weight-scan finding (a fingerprint that no longer matches the load).
    Replays that differed are confirmed too (an exact replay has no rounding envelope to sit inside), and so is a
    spot check past its rigorous bound."""
    if ev.detector in ("weights", "replay", "quantization", "collective", "spot", "kv_transfer", "alltoall"):
        return True
    rec = (ev.detail or {}).get("recheck") or {}
    return rec.get("verdict") in CONFIRMING_RECHECKS


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
        self.captures: list[dict] = []       # captured alarms with their float64 rechecks

    def mark_step(self, step: int) -> None:
        self.step = step

    def attach_weight_scan(self, scan, budget_mb: float = 256.0) -> None:
        """Scan `budget_mb` of weights (serve.weights.WeightScan) at every poll."""
        self.weight_scan = scan
        self.scan_budget_mb = budget_mb

    def poll(self, reset: bool = True, wait: bool = True) -> list[SDCEvent]:
        """Read the state rows, record events for alarms, reset the rows.

        wait=True: read everything up to now (one device-to-host copy that waits for the stream), together with any
        read still in flight. wait=False never waits for the GPU: it turns the results of the previous poll's read
        into events if that read has landed, and starts the next read (a device snapshot and a pinned-memory copy
        ordered after the work queued so far). Results therefore arrive one poll late, as in the reference's
        poll (src/sdcguard/serve.py:1090-1129)."""
        with nvtx_range("sdcguard.poll"):
            return self._poll(reset, wait)

    def _poll(self, reset: bool, wait: bool) -> list[SDCEvent]:
        events: list[SDCEvent] = []
        pending = getattr(self, "_pending", None)
        if pending is not None and (wait or pending.ready()):
            events += self._fold(pending.result(wait=True))
            self._pending = pending = None
        if wait:
            events += self._fold(self.model.state.read(reset=reset))
            events += self._runtime_errors()
            self._attach_capture(events)
        elif pending is None:
            self._pending = self.model.state.read_async(reset=reset)
        if self.weight_scan is not None:
            for ev in self.weight_scan.poll(self.scan_budget_mb, step=self.step):
                self.log.add(ev)
                events.append(ev)
                if self.on_alert:
                    self.on_alert(ev)
        return events

    def _attach_capture(self, events: list[SDCEvent]) -> None:
        """The device's captured alarm (the first GEMM alarm since the last read: its input row, its block sums,
        the sums it was judged against) goes into the detail of the checksum event of the same layer, with the
        float64 recheck against the layer's weights (weights changed / output wrong / expected side wrong /
        not reproduced)."""
        from ..ops import gemm
        dev = getattr(self.model, "device", None)
        if dev is None or torch.device(dev).type != "cuda":
            return
        cap = gemm.read_capture(torch.device(dev))
        if cap is None:
            return
        slot = self.model.state.slot_of(cap["state_row"])
        if slot is None:       # an alarm of another table's GEMM (another model or tool on this device)
            return
        cw = getattr(self.model, "slot_weights", {}).get(slot)
        rec = gemm.recheck_capture(cap, cw) if cw is not None and cw.k == cap["k"] else None
        name = self.model.state.names[slot]
        kept = {k: v for k, v in cap.items() if k != "x_row"}
        for ev in events:
            if ev.detector == "checksum" and ev.detail.get("layer") == name:
                ev.detail["captured"] = kept
                ev.detail["recheck"] = rec
                self.captures.append({"layer": name, "captured": kept, "recheck": rec, "x_row": cap["x_row"]})
                return
        self.captures.append({"layer": name, "captured": kept, "recheck": rec, "x_row": cap["x_row"]})

    def _runtime_errors(self) -> list[SDCEvent]:
        """A kernel whose bounded wait ran out (its error word is set): reported as an event of its own, and the
        GEMM band counters it may have left raised are cleared (ops.gemm.take_errors)."""
        from ..ops import gemm
        dev = getattr(self.model, "device", None)
        if dev is None or torch.device(dev).type != "cuda":
            return []
        code = gemm.take_errors(torch.device(dev))
        if not code:
            return []
        if self._identity is None:
            self._identity = device_identity(dev)
        ev = SDCEvent(detector="runtime", step=self.step,
                      detail={"error_code": code, "what": gemm.ERROR_NAMES.get(code, "unknown")}, identity=self._identity)
        self.log.add(ev)
        if self.on_alert:
            self.on_alert(ev)
        return [ev]

    def _fold(self, rows) -> list[SDCEvent]:
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
                det = ("checksum" if "GEMM" in r["name"] else "collective" if "collective" in r["name"]
                       else "spot" if "spot" in r["name"] else "quantization" if ".quant" in r["name"]
                       else "replay")
                detail = {"layer": r["name"], "z": z, "noise": r["noise"], "flat": r["flat"]}
                if "row" in r:
                    detail.update({k: r[k] for k in ("row", "block", "signed", "peer") if k in r})
                ev = SDCEvent(detector=det, step=self.step, detail=detail, identity=self._identity)
                self.log.add(ev)
                events.append(ev)
                if self.on_alert:
                    self.on_alert(ev)
        return events

    def coverage_report(self) -> dict:
        """ops / ops_checked: the checks that run on every step they cover (ABFT GEMMs, replays, transfers) and how
        many of them have run. The spot check takes one projection per prefill step in turn, so its slots are
        counted apart (sampled_ops, sampled_ops_run): a short window leaves some of them unvisited by design."""
        every = {n: t for n, t in self.totals.items() if "spot check" not in n}
        sampled = {n: t for n, t in self.totals.items() if "spot check" in n}
        checked = sum(1 for t in every.values() if t["checks"] > 0)
        quant = {n: t for n, t in self.totals.items() if ".quant" in n}
        return {"ops": len(every), "ops_checked": checked, "sampled_ops": len(sampled),
                "sampled_ops_run": sum(1 for t in sampled.values() if t["checks"] > 0),
                "checks": sum(t["checks"] for t in self.totals.values()),
                "unjudged": sum(t["unjudged"] for t in self.totals.values()),
                "alarms": sum(t["alarms"] for t in self.totals.values()),
                "fp8_calls_judged": sum(t["checks"] for t in quant.values()),
                "fp8_findings": sum(t["alarms"] for t in quant.values()),
                "alerts": len(self.log.events),
                "confirmed_alerts": sum(1 for e in self.log.events if confirmed(e)),
                "worst_clean_z": max((t["worst_z"] for t in self.totals.values() if t["alarms"] == 0), default=0.0)}

    def worst_z(self) -> float:
        return max((t["worst_z"] for t in self.totals.values()), default=0.0)
