"""Health events for NVIDIA NVSentinel (the Kubernetes GPU fault pipeline): this package's findings as one more
monitor, agent "sdcguard", check "GpuComputeCorrectness".

  * An alert from a job (an ABFT, replay, spot, transfer, canary or replica detector; utils.events.SDCEvent) is a
    lead, not a verdict: it is sent unhealthy but not fatal, with processing strategy STORE_AND_ANALYSE and no
    recommended action, one event per GPU and detector with the count, first and last time and worst score.
  * A `sdcguard check` result of a node's GPU: FAIL is unhealthy, PASS healthy (clearing an earlier FAIL of the
    same check and GPU), both STORE_AND_ANALYSE unless `remediate` is set, when a FAIL goes as fatal
    EXECUTE_REMEDIATION recommending RUN_FIELDDIAG and a PASS as EXECUTE_REMEDIATION healthy. Anything else
    (an incomplete run) is not sent.

A GPU is named by its UUID and its PCI address in NVSentinel's form (0000:1b:00.0), never by an index. Events are
sent as one HealthEvents batch per call over NVSentinel's node socket (gRPC, unary
/datamodels.PlatformConnector/HealthEventOccurredV1), with the projected service-account token as a bearer token
when one is mounted (read again for every call); UNAVAILABLE and DEADLINE_EXCEEDED are retried with backoff, any
other status is NVSentinel's answer and is reported. Messages are written with this module's own protobuf wire
writer, so no generated code is needed; the message and field numbers are NVSentinel's health_event.proto.

    sdcguard nvsentinel check.json [--remediate]      a node's check result
    sdcguard nvsentinel alerts.jsonl                  a job's alert log
    sdcguard nvsentinel ... --dry-run                 print the events, send nothing

In a job: `SDCGuard(on_alert=Publisher())` or `ServeGuard(..., on_alert=Publisher())` sends alerts from a background
thread, at most one per GPU and detector every `min_interval` seconds; failures are counted, never raised.

Reference: src/sdcguard/nvsentinel.py (`encode_event` :86, `from_check` :172, `from_alerts` :212, `send` :276,
`Publisher` :319); the event semantics, field numbers and socket / method / token paths are kept so both tools
feed the same NVSentinel rules.
"""
from __future__ import annotations

import argparse
import json
import os
import socket
import threading
import time
from dataclasses import dataclass, field
from typing import Iterable, Optional

SOCKET = "/var/run/nvsentinel.sock"
TOKEN = "/var/run/secrets/nvsentinel/platform-connector/token"
METHOD = "/datamodels.PlatformConnector/HealthEventOccurredV1"
AGENT = "sdcguard"
CHECK = "GpuComputeCorrectness"
STRATEGY = {"UNSPECIFIED": 0, "EXECUTE_REMEDIATION": 1, "STORE_ONLY": 2, "STORE_AND_ANALYSE": 3}
ACTION = {"NONE": 0, "COMPONENT_RESET": 2, "CONTACT_SUPPORT": 5, "RUN_FIELDDIAG": 6, "RESTART_VM": 15,
          "RESTART_BM": 24, "REPLACE_VM": 25, "RUN_DCGMEUD": 26, "CUSTOM": 27, "UNKNOWN": 99}
DETECTOR_CODES = {"checksum": "SDCGUARD_CHECKSUM", "replay": "SDCGUARD_REPLAY_MISMATCH", "spot": "SDCGUARD_SPOT_CHECK",
                  "collective": "SDCGUARD_TRANSFER_SEAL", "kv_transfer": "SDCGUARD_KV_PAGE_CHECKSUM",
                  "alltoall": "SDCGUARD_TRANSFER_SEAL", "canary": "SDCGUARD_CANARY_MISMATCH",
                  "replica": "SDCGUARD_REPLICA_DIVERGENCE", "recompute": "SDCGUARD_RECOMPUTE_MISMATCH",
                  "weights": "SDCGUARD_WEIGHT_FINGERPRINT", "runtime": "SDCGUARD_KERNEL_WAIT_TIMEOUT"}


# ------------------------------------------------------------------------------------------ protobuf wire writer
class Wire:
    """A proto3 message being written: fields are appended in the caller's (field-number) order; default values
    (0, False, empty) are skipped, as a proto3 serializer does."""

    def __init__(self):
        self.buf = bytearray()

    @staticmethod
    def varint(n: int) -> bytes:
        n &= (1 << 64) - 1            # negative int64 / enum values: ten bytes of two's complement
        out = bytearray()
        while n >= 0x80:
            out.append((n & 0x7F) | 0x80)
            n >>= 7
        out.append(n)
        return bytes(out)

    def _tag(self, num: int, wt: int) -> None:
        self.buf += self.varint((num << 3) | wt)

    def uint(self, num: int, v) -> "Wire":
        if v:
            self._tag(num, 0)
            self.buf += self.varint(int(v))
        return self

    def flag(self, num: int, v) -> "Wire":
        return self.uint(num, 1 if v else 0)

    def raw(self, num: int, data: bytes, keep_empty: bool = False) -> "Wire":
        if data or keep_empty:
            self._tag(num, 2)
            self.buf += self.varint(len(data)) + data
        return self

    def text(self, num: int, s) -> "Wire":
        return self.raw(num, str(s).encode()) if s else self

    def sub(self, num: int, w: "Wire") -> "Wire":
        return self.raw(num, bytes(w.buf), keep_empty=True)

    def bytes(self) -> bytes:
        return bytes(self.buf)


@dataclass
class HealthEvent:
    message: str
    healthy: bool
    entities: list                          # [(type, value)] e.g. ("GPU_UUID", "GPU-..."), ("PCI", "0000:1b:00.0")
    fatal: bool = False
    action: str = "NONE"
    codes: list = field(default_factory=list)
    metadata: dict = field(default_factory=dict)
    when: float = field(default_factory=time.time)
    node: str = ""
    strategy: str = "STORE_AND_ANALYSE"
    component: str = "GPU"

    def encode(self) -> bytes:
        """health_event.proto HealthEvent: 1 version, 2 agent, 3 componentClass, 4 checkName, 5 isFatal,
        6 isHealthy, 7 message, 8 recommendedAction, 9 errorCode (repeated), 10 entitiesImpacted (Entity: 1 type,
        2 value), 11 metadata (map entries: 1 key, 2 value, by key), 12 generatedTimestamp (1 seconds, 2 nanos),
        13 nodeName, 16 processingStrategy."""
        w = Wire().uint(1, 1).text(2, AGENT).text(3, self.component).text(4, CHECK)
        w.flag(5, self.fatal).flag(6, self.healthy).text(7, self.message).uint(8, ACTION[self.action])
        for c in self.codes:
            w.raw(9, str(c).encode(), keep_empty=True)
        for typ, val in self.entities:
            w.sub(10, Wire().text(1, typ).text(2, val))
        for k in sorted(self.metadata):
            w.sub(11, Wire().raw(1, str(k).encode(), True).raw(2, str(self.metadata[k]).encode(), True))
        sec = int(self.when)
        nanos = min(int(round((self.when - sec) * 1e9)), 999_999_999)
        w.sub(12, Wire().uint(1, sec).uint(2, nanos))
        w.text(13, self.node).uint(16, STRATEGY[self.strategy])
        return w.bytes()

    def as_dict(self) -> dict:
        return {"agent": AGENT, "checkName": CHECK, "componentClass": self.component, "isFatal": self.fatal,
                "isHealthy": self.healthy, "message": self.message, "recommendedAction": self.action,
                "errorCode": self.codes, "entitiesImpacted": [{"entityType": t, "entityValue": v}
                                                               for t, v in self.entities],
                "metadata": self.metadata, "generatedTimestamp": self.when, "nodeName": self.node,
                "processingStrategy": self.strategy}


def encode_batch(events: Iterable[HealthEvent]) -> bytes:
    """HealthEvents: 1 version, 2 events (repeated)."""
    w = Wire().uint(1, 1)
    for e in events:
        w.raw(2, e.encode(), keep_empty=True)
    return w.bytes()


# ------------------------------------------------------------------------------------------ events from findings
def pci_entity(bus: Optional[str]) -> Optional[str]:
    """nvidia-smi's 00000000:1B:00.0 as NVSentinel writes PCI entities: four domain digits, lower case."""
    if not bus or not isinstance(bus, str):
        return None
    parts = bus.strip().split(":")
    if len(parts) != 3:
        return bus.strip().lower()
    return f"{parts[0][-4:]}:{parts[1]}:{parts[2]}".lower()


def _entities(uuid: Optional[str], bus: Optional[str]) -> list:
    out = []
    pci = pci_entity(bus)
    if pci:
        out.append(("PCI", pci))
    if uuid:
        out.append(("GPU_UUID", str(uuid)))
    return out


def node_name(given: Optional[str] = None) -> str:
    """The Kubernetes node: given, else NODE_NAME (the downward API), else this host outside a pod ("" inside a pod
    without NODE_NAME: a pod's hostname is not the node's)."""
    if given:
        return given
    if os.environ.get("NODE_NAME"):
        return os.environ["NODE_NAME"]
    return "" if os.environ.get("KUBERNETES_SERVICE_HOST") else socket.gethostname()


def _short(v, n: int = 256) -> str:
    s = "" if v is None else str(v)
    return s if len(s) <= n else s[: n - 3] + "..."


def from_check(result: dict, node: str = "", remediate: bool = False) -> tuple:
    """(event or None, reason) for a check result: {"result": PASS/FAIL, "gpu_uuid", "pci_bus_id", "device", ...}
    (`sdcguard check --json`)."""
    from .. import __version__
    r = str(result.get("result") or "")
    if r not in ("PASS", "FAIL"):
        return None, f"{r or 'no result'}: says nothing about the GPU's health"
    uuid = result.get("gpu_uuid") or (result.get("gpu") or {}).get("uuid")
    if not uuid:
        return None, "the result does not name its GPU's UUID"
    healthy = r == "PASS"
    fatal = (not healthy) and remediate
    msg = f"sdcguard check {r} on {result.get('device') or 'GPU'} {uuid}"
    if not healthy:
        msg += f": {result.get('gemm_wrong', 0)} wrong GEMM results, {result.get('copies_wrong', 0)} wrong copies"
    meta = {"sdcguard_version": __version__, "source": "sdcguard check", "result": r,
            "gpu_name": result.get("device"), "worst_z": result.get("worst_z")}
    ev = HealthEvent(message=_short(msg, 1024), healthy=healthy, fatal=fatal,
                     entities=_entities(uuid, result.get("pci_bus_id")),
                     action="RUN_FIELDDIAG" if fatal else "NONE", codes=[] if healthy else ["SDCGUARD_CHECK_FAIL"],
                     metadata={k: _short(v) for k, v in meta.items() if v not in (None, "")}, node=node,
                     strategy="EXECUTE_REMEDIATION" if remediate else "STORE_AND_ANALYSE")
    return ev, None


def from_alerts(alerts: Iterable[dict], node: str = "", host: Optional[str] = None) -> tuple:
    """(events, skipped) for SDCEvent dicts (a JSONL alert log): one event per (GPU, detector) of this host."""
    from .. import __version__
    host = host or socket.gethostname()
    groups: dict = {}
    skipped = []
    for a in alerts:
        ident = a.get("identity") or {}
        det = str(a.get("detector") or "checksum")
        if not ident.get("gpu_uuid"):
            skipped.append(f"{det} alert without a GPU UUID")
            continue
        if ident.get("host") and ident["host"] != host:
            skipped.append(f"{det} alert of host {ident['host']} (send it from that node)")
            continue
        g = groups.setdefault((ident["gpu_uuid"], det), {"ident": ident, "n": 0, "times": [], "z": None,
                                                         "where": None})
        g["n"] += 1
        if isinstance(a.get("time"), (int, float)):
            g["times"].append(float(a["time"]))
        d = a.get("detail") or {}
        z = d.get("z")
        if isinstance(z, (int, float)):
            g["z"] = z if g["z"] is None else max(g["z"], z)
        g["where"] = g["where"] or d.get("layer")
    out = []
    for (uuid, det), g in sorted(groups.items()):
        ident, ts = g["ident"], g["times"]
        meta = {"sdcguard_version": __version__, "source": "in-job alert", "detector": det, "alerts": g["n"],
                "first_alert": _iso(min(ts)) if ts else None, "last_alert": _iso(max(ts)) if ts else None,
                "worst_z": g["z"], "where": g["where"], "gpu_name": ident.get("gpu_name"), "verified": "false"}
        out.append(HealthEvent(
            message=_short(f"sdcguard: {g['n']} {det} alert{'s' if g['n'] != 1 else ''} on "
                           f"{ident.get('gpu_name') or 'GPU'} {uuid}; a lead to confirm with sdcguard check or "
                           "casefile, not a verdict", 1024),
            healthy=False, fatal=False, entities=_entities(uuid, ident.get("pci_bus_id")),
            codes=[DETECTOR_CODES.get(det, f"SDCGUARD_{det.upper()}")],
            metadata={k: _short(v) for k, v in meta.items() if v not in (None, "")},
            when=max(ts) if ts else time.time(), node=node))
    return out, skipped


def _iso(t: float) -> str:
    return time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime(t))


# ------------------------------------------------------------------------------------------ sending
class SendError(RuntimeError):
    pass


def send(events: list, socket_path: str = SOCKET, token_file: Optional[str] = None, timeout: float = 10.0,
         retries: int = 4, backoff: float = 1.0) -> None:
    """One batch (NVSentinel accepts or refuses a batch whole); raises SendError with the reason."""
    if not events:
        return
    if not os.path.exists(socket_path):
        raise SendError(f"no NVSentinel socket at {socket_path} (platform connector not running on this node, or "
                        "its hostPath not mounted here)")
    try:
        import grpc
    except ImportError as e:
        raise SendError("sending to NVSentinel needs grpcio") from e
    if token_file is None and os.path.exists(TOKEN):
        token_file = TOKEN
    body = encode_batch(events)
    again = {grpc.StatusCode.UNAVAILABLE, grpc.StatusCode.DEADLINE_EXCEEDED}
    last = "no attempt"
    with grpc.insecure_channel(f"unix://{socket_path}") as ch:
        rpc = ch.unary_unary(METHOD, request_serializer=None, response_deserializer=None)
        for attempt in range(max(1, retries)):
            md = None
            if token_file:
                with open(token_file) as f:
                    tok = f.read().strip()
                if not tok:
                    raise SendError(f"token file {token_file} is empty")
                md = (("authorization", f"Bearer {tok}"),)
            try:
                rpc(body, timeout=timeout, metadata=md)
                return
            except grpc.RpcError as e:
                code = e.code() if hasattr(e, "code") else None
                last = f"{getattr(code, 'name', code)}: {e.details() if hasattr(e, 'details') else e}"
                if code not in again:
                    raise SendError(f"NVSentinel refused the events ({last})") from e
            time.sleep(backoff * (2 ** attempt))
    raise SendError(f"NVSentinel did not answer ({last})")


class Publisher:
    """An on_alert callback: each SDCEvent about this host's GPUs goes to NVSentinel from a background thread, at
    most one per (GPU, detector) every `min_interval` seconds. Failures are counted, never raised."""

    def __init__(self, socket_path: str = SOCKET, token_file: Optional[str] = None, node: Optional[str] = None,
                 min_interval: float = 300.0, timeout: float = 5.0, sender=None):
        self.socket_path, self.token_file, self.timeout = socket_path, token_file, timeout
        self.node = node_name(node)
        self.min_interval = min_interval
        self._send = sender or send
        self._last: dict = {}
        self._lock = threading.Lock()
        self._threads: list = []
        self.sent = self.failed = self.skipped = 0
        self.errors: list = []

    def __call__(self, ev) -> None:
        d = ev if isinstance(ev, dict) else {"detector": ev.detector, "step": ev.step, "detail": ev.detail,
                                              "identity": ev.identity, "time": ev.time}
        events, skipped = from_alerts([d], node=self.node)
        if not events:
            with self._lock:
                self.skipped += 1
            return
        key = (d["identity"].get("gpu_uuid"), d.get("detector"))
        now = time.monotonic()
        with self._lock:
            if key in self._last and now - self._last[key] < self.min_interval:
                self.skipped += 1
                return
            self._last[key] = now
        t = threading.Thread(target=self._deliver, args=(events,), daemon=True)
        t.start()
        self._threads.append(t)

    def _deliver(self, events) -> None:
        try:
            self._send(events, socket_path=self.socket_path, token_file=self.token_file, timeout=self.timeout)
            with self._lock:
                self.sent += len(events)
        except Exception as e:  # noqa: BLE001  (an alert must not stop the job)
            with self._lock:
                self.failed += len(events)
                self.errors.append(str(e))

    def flush(self, timeout: float = 30.0) -> None:
        for t in list(self._threads):
            t.join(timeout)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="sdcguard nvsentinel", description=__doc__.split("\n\n")[0])
    ap.add_argument("path", help="a check result (.json) or an alert log (.jsonl)")
    ap.add_argument("--remediate", action="store_true", help="a FAIL asks NVSentinel for remediation")
    ap.add_argument("--dry-run", action="store_true")
    ap.add_argument("--socket", default=SOCKET)
    ap.add_argument("--token-file")
    ap.add_argument("--node")
    a = ap.parse_args(argv)
    node = node_name(a.node)
    events, skipped = [], []
    with open(a.path) as f:
        text = f.read()
    if a.path.endswith(".jsonl"):
        rows = [json.loads(line) for line in text.splitlines() if line.strip()]
        events, skipped = from_alerts(rows, node=node)
    else:
        ev, why = from_check(json.loads(text), node=node, remediate=a.remediate)
        events, skipped = ([ev], []) if ev else ([], [why])
    if a.dry_run or not events:
        print(json.dumps({"events": [e.as_dict() for e in events], "skipped": skipped}, indent=1))
        return 0
    try:
        send(events, socket_path=a.socket, token_file=a.token_file)
    except SendError as e:
        print(f"sdcguard nvsentinel: {e}")
        return 2
    print(json.dumps({"sent": len(events), "skipped": skipped}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
