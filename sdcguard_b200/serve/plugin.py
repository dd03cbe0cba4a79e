"""Plugin hooks of the serving engine: the points where the guard attaches to a serving runtime, as the
reference attaches to vLLM (src/sdcguard/vllm_plugin.py: `register` :2239 patches weight loading :2315, the linear
`apply` :2344, `execute_model` :2430-2501 (mark_step, poll every SDCGUARD_POLL_EVERY steps), `load_model` :2410;
SDCGUARD_REQUIRE refuses to serve unchecked :500-547; alerts are attributed to requests :677).

Here the engine is this package's own, so the hooks are explicit:

    hooks = register(engine, poll_every=16, require=True, on_alert=chain(webhook, metrics.on_event))
    engine.generate(...)                       # every prefill batch / decode step calls hooks.after_step
    hooks.report()                             # coverage, alarms, attributed requests

  * weights_loaded: runs once at registration (builds the weight scan, collects the stack identity);
  * after_step(kind, rows_to_requests): counts steps and polls the guard every `poll_every` steps without waiting
    for the GPU (the results of a poll's read are turned into alerts at the next poll), or waiting when
    `poll_seconds` have passed since the last read; attributes each alarm's row to the request it belongs to;
  * require: refuse to serve a model whose GEMMs are not checked (the SDCGUARD_REQUIRE rule).
Environment: SDCGUARD_POLL_EVERY (default 16), SDCGUARD_POLL_SECONDS (default 2), SDCGUARD_REQUIRE (1: require),
SDCGUARD_SCAN_MB (weight scan budget per poll, default 0 = off).
"""
from __future__ import annotations

import os
import time
from typing import Callable, Optional

from ..utils import stack as stack_mod
from ..utils.events import SDCEvent


class UncheckedServingRefused(RuntimeError):
    pass


class PluginHooks:
    def __init__(self, engine, poll_every: int = 16, on_alert: Optional[Callable[[SDCEvent], None]] = None,
                 poll_seconds: float = 2.0):
        self.engine = engine
        self.guard = engine.guard
        self.poll_every = max(1, poll_every)
        self.poll_seconds = poll_seconds
        self._last_poll = time.monotonic()
        self._inflight_rows: list[tuple[str, list[int]]] = []   # rows of the steps the pending read covers
        self.on_alert = on_alert
        self.steps = 0
        self.polls = 0
        self.alerts: list[dict] = []
        self._rows: list[tuple[str, list[int]]] = []     # rows -> request of the steps since the last poll
        self.stack: dict = {}
        self.weight_scan = None
        self.step_hooks: list[Callable] = []

    def weights_loaded(self, scan_mb: float = 0.0) -> None:
        model = self.engine.model
        if scan_mb > 0:
            from .weights import WeightScan
            named = [("embed", model.embed)] + [(f"layers.{i}.{n}", getattr(lw, n))
                                                for i, lw in enumerate(model.layers)
                                                for n in ("qkv", "o", "gate_up", "down")
                                                if getattr(lw, n, None) is not None]
            self.weight_scan = WeightScan(named)
            self.guard.attach_weight_scan(self.weight_scan, scan_mb)
        self.stack = stack_mod.collect(model, self.engine, self.weight_scan)

    def after_step(self, kind: str, rows_to_requests: list[int]) -> None:
        self.steps += 1
        self.guard.mark_step(self.engine.step_counter)
        self._rows.append((kind, list(rows_to_requests)))
        for h in self.step_hooks:
            h(kind, self.steps)
        late = time.monotonic() - self._last_poll >= self.poll_seconds
        if self.steps % self.poll_every == 0 or late:
            self.poll(wait=late)

    def poll(self, wait: bool = True) -> list[SDCEvent]:
        """wait=False: alerts from the previous poll's read if it has landed, and a new read started (never waits
        for the GPU); wait=True: everything up to now."""
        self.polls += 1
        self._last_poll = time.monotonic()
        events = self.guard.poll(wait=wait)
        windows = self._inflight_rows + self._rows
        for ev in events:
            req = None
            row = ev.detail.get("row")
            if row is not None:
                for _, mapping in reversed(windows):
                    if 0 <= row < len(mapping):
                        req = mapping[row]
                        break
            self.alerts.append({"detector": ev.detector, "step": ev.step, "detail": ev.detail, "request": req})
            if self.on_alert:
                self.on_alert(ev)
        self._inflight_rows = [] if wait else list(self._rows)
        self._rows.clear()
        return events

    def report(self) -> dict:
        return {"steps": self.steps, "polls": self.polls, "alerts": self.alerts,
                "coverage": self.guard.coverage_report(), "stack": self.stack}


def register(engine, poll_every: Optional[int] = None, require: Optional[bool] = None,
             on_alert: Optional[Callable[[SDCEvent], None]] = None, scan_mb: Optional[float] = None) -> PluginHooks:
    poll_every = int(os.environ.get("SDCGUARD_POLL_EVERY", "16")) if poll_every is None else poll_every
    poll_seconds = float(os.environ.get("SDCGUARD_POLL_SECONDS", "2"))
    require = os.environ.get("SDCGUARD_REQUIRE", "0") == "1" if require is None else require
    scan_mb = float(os.environ.get("SDCGUARD_SCAN_MB", "0")) if scan_mb is None else scan_mb
    if require and not getattr(engine.model, "checked", False):
        raise UncheckedServingRefused("SDCGUARD_REQUIRE is set and the model's GEMMs are not checked")
    hooks = PluginHooks(engine, poll_every, on_alert, poll_seconds)
    hooks.weights_loaded(scan_mb)
    engine.hooks = hooks
    return hooks
