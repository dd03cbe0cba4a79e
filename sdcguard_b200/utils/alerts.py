"""Alert delivery and metrics: webhooks (Slack, Discord or plain JSON) posted from a background thread so a slow
endpoint never stalls the serving loop, and Prometheus metrics per detector.

    hooks = Webhook("https://hooks.slack.com/...", kind="slack")
    metrics = Metrics()                          # prometheus_client registry; metrics.serve(9400) to expose
    guard = ServeGuard(model, on_alert=chain(hooks, metrics.on_event))

Reference: `Webhook` (src/sdcguard/alerts.py:97), `Metrics` (:216), `chain` (:186).
"""
from __future__ import annotations

import json
import logging
import queue
import threading
import urllib.request
from typing import Callable, Optional

from .events import SDCEvent

log = logging.getLogger("sdcguard")


def text(ev: SDCEvent) -> str:
    d = ev.detail
    where = ", ".join(f"{k}={d[k]}" for k in ("layer", "weight", "block", "row", "suspect_ranks", "phase") if k in d)
    ident = ev.identity or {}
    gpu = ident.get("gpu_uuid") or ident.get("device") or "?"
    return f"sdcguard: {ev.detector} alarm at step {ev.step} on {ident.get('host', '?')} GPU {gpu}: {where}"


class Webhook:
    def __init__(self, url: str, kind: str = "json", timeout: float = 5.0, max_queue: int = 1000):
        if kind not in ("json", "slack", "discord"):
            raise ValueError("kind must be json, slack or discord")
        self.url, self.kind, self.timeout = url, kind, timeout
        self.q: queue.Queue = queue.Queue(maxsize=max_queue)
        self.sent = 0
        self.failed = 0
        self.dropped = 0
        self.skipped = 0
        self._t = threading.Thread(target=self._run, daemon=True, name="sdcguard-webhook")
        self._t.start()

    def payload(self, ev: SDCEvent) -> dict:
        if self.kind == "slack":
            return {"text": text(ev)}
        if self.kind == "discord":
            return {"content": text(ev)}
        return json.loads(ev.to_json())

    def __call__(self, ev: SDCEvent) -> None:
        if ev.detail.get("reporter") is False:      # a cross-rank vote's finding: one rank posts it, not every rank
            self.skipped += 1
            return
        try:
            self.q.put_nowait(ev)
        except queue.Full:
            self.dropped += 1

    def _run(self) -> None:
        while True:
            ev = self.q.get()
            if ev is None:
                return
            data = json.dumps(self.payload(ev)).encode()
            req = urllib.request.Request(self.url, data=data, headers={"Content-Type": "application/json"})
            try:
                with urllib.request.urlopen(req, timeout=self.timeout):
                    self.sent += 1
            except Exception as e:  # noqa: BLE001  delivery is best effort; the event stays in the log
                self.failed += 1
                if self.failed == 1:
                    log.warning("sdcguard: webhook delivery failed (%s)", e)

    def close(self, timeout: float = 5.0) -> None:
        self.q.put(None)
        self._t.join(timeout)


def chain(*handlers: Optional[Callable[[SDCEvent], None]]) -> Callable[[SDCEvent], None]:
    hs = [h for h in handlers if h is not None]

    def run(ev: SDCEvent) -> None:
        for h in hs:
            try:
                h(ev)
            except Exception as e:  # noqa: BLE001  one failing handler must not hide the alarm from the others
                log.warning("sdcguard: alert handler failed (%s)", e)
    return run


class Metrics:
    """Prometheus counters and gauges: alarms per detector, checks run, worst clean score, stack identity."""

    def __init__(self, registry=None, prefix: str = "sdcguard"):
        from prometheus_client import CollectorRegistry, Counter, Gauge
        self.registry = registry or CollectorRegistry()
        self.alarms = Counter(f"{prefix}_alarms", "SDC alarms", ["detector"], registry=self.registry)
        self.checks = Counter(f"{prefix}_checks", "checks executed", ["kind"], registry=self.registry)
        self.worst = Gauge(f"{prefix}_worst_clean_z", "worst score of a clean check", registry=self.registry)
        self.unjudged = Counter(f"{prefix}_unjudged", "checksums left unjudged", registry=self.registry)
        self.info = Gauge(f"{prefix}_stack_info", "serving stack identity", ["key", "value"], registry=self.registry)

    def on_event(self, ev: SDCEvent) -> None:
        self.alarms.labels(ev.detector).inc()

    def observe_coverage(self, report: dict, kind: str = "serve") -> None:
        self.checks.labels(kind).inc(report.get("checks", 0))
        self.unjudged.inc(report.get("unjudged", 0))
        self.worst.set(report.get("worst_clean_z", 0.0))

    def publish_stack(self, stack: dict) -> None:
        for k, v in stack.items():
            if isinstance(v, (str, int, float, bool)):
                self.info.labels(k, str(v)).set(1)

    def text(self) -> bytes:
        from prometheus_client import generate_latest
        return generate_latest(self.registry)

    def serve(self, port: int, addr: str = "127.0.0.1") -> None:
        from prometheus_client import start_http_server
        start_http_server(port, addr=addr, registry=self.registry)
