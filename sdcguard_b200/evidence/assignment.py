"""Inspection of the recorded allocator-to-request mapping of a run of this engine: which KV pages each request was
assigned, shared and freed, and whether any page was assigned to a second request while the first still held it.

    python -m sdcguard_b200.evidence.assignment inspect lifetime.jsonl [--json]
    python -m sdcguard_b200.evidence.assignment packet lifetime.jsonl --out PACKET.json
    python -m sdcguard_b200.evidence.assignment verify PACKET.json
    sdcguard assignment ...

The input is the lifetime event stream (`lifetime.adapter.EventSink`: alloc, share, free, ...). Ownership is
replayed in order: alloc gives a page to its owner with a new generation, share adds a reader of that generation,
free ends it. Findings: a page allocated while live (double assignment), a share or free naming a generation that is
not the live one, and pages never freed (reported, not a violation: the run may have ended with requests live).
A packet holds the events, their digest and the report; verify re-derives the report from the packet's own events.
It reads records only: no engine or request is started, and it says nothing about traffic the events do not record.

Reference: src/sdcguard/assignment_report.py:1-10 (`parse_records`, `inspect_payload`, `render_report`,
`create_packet`, `verify_packet`).
"""
from __future__ import annotations

import argparse
import hashlib
import json
import sys

from . import catalog

SCHEMA = "sdcguard_b200.assignment-packet.v1"
MAX_EVENTS = 10_000_000


def parse_records(path: str) -> list[dict]:
    out = []
    with open(path) as f:
        for i, line in enumerate(f):
            if not line.strip():
                continue
            e = json.loads(line)
            if not isinstance(e, dict) or "ev" not in e:
                raise ValueError(f"line {i + 1}: not an event")
            out.append(e)
            if len(out) > MAX_EVENTS:
                raise ValueError("too many events")
    return out


class Ownership:
    """Replayed page ownership: region -> (owner, generation, readers) while live."""

    def __init__(self):
        self.live: dict = {}
        self.gen: dict = {}
        self.issues: list[dict] = []
        self.per_request: dict = {}

    def _req(self, r):
        return self.per_request.setdefault(r, {"allocated": 0, "shared": 0, "freed": 0})

    def apply(self, i: int, e: dict) -> None:
        k = e["ev"]
        if k == "alloc":
            reg = tuple(e["region"])
            if reg in self.live:
                self.issues.append({"event": i, "kind": "double_assignment", "region": list(reg),
                                    "holder": self.live[reg][0], "new_owner": e["owner"]})
            self.gen[reg] = self.gen.get(reg, 0) + 1
            self.live[reg] = (e["owner"], self.gen[reg], set())
            self._req(e["owner"])["allocated"] += 1
        elif k in ("share", "free"):
            reg = tuple(e["region"])
            cur = self.live.get(reg)
            if cur is None or cur[1] != e.get("gen"):
                self.issues.append({"event": i, "kind": f"{k}_of_stale_generation", "region": list(reg),
                                    "gen": e.get("gen"), "live_gen": None if cur is None else cur[1]})
                return
            if k == "share":
                cur[2].add(e["request"])
                self._req(e["request"])["shared"] += 1
            else:
                self._req(cur[0])["freed"] += 1
                del self.live[reg]

    def holders(self, reg: tuple):
        cur = self.live.get(reg)
        return None if cur is None else (cur[0], cur[1], cur[2])


def inspect_payload(events: list[dict]) -> dict:
    own = Ownership()
    for i, e in enumerate(events):
        own.apply(i, e)
    bad = [x for x in own.issues if x["kind"] == "double_assignment"]
    f = catalog.finding("assignment.exclusive", "violated" if bad else "satisfied",
                        f"{len(bad)} page(s) assigned to a second request while held" if bad else
                        "no page was assigned to two live requests", "recorded lifetime events",
                        {"events": len(events), "requests": len(own.per_request)})
    return {"schema": "sdcguard_b200.assignment-report.v1", "events": len(events), "requests": own.per_request,
            "issues": own.issues, "live_at_end": len(own.live), "findings": [f],
            "verdict": "FAIL" if bad else ("HOLD" if own.issues else "PASS"),
            "scope": "the recorded events of one run; not unrecorded traffic"}


def render_report(r: dict) -> str:
    lines = [f"assignment: {r['verdict']} ({r['events']} events, {len(r['requests'])} requests, "
             f"{r['live_at_end']} pages live at the end)"]
    lines += [f"  {x['kind']} at event {x['event']}: region {x['region']}" for x in r["issues"][:50]]
    return "\n".join(lines)


def _digest(events) -> str:
    return hashlib.sha256(json.dumps(events, sort_keys=True, separators=(",", ":")).encode()).hexdigest()


def create_packet(events: list[dict]) -> dict:
    return {"schema": SCHEMA, "events": events, "events_sha256": _digest(events), "report": inspect_payload(events)}


def verify_packet(p: dict) -> list[str]:
    if not isinstance(p, dict) or p.get("schema") != SCHEMA:
        return [f"not a {SCHEMA} packet"]
    bad = []
    if _digest(p.get("events")) != p.get("events_sha256"):
        bad.append("events digest differs")
    if inspect_payload(p["events"]) != p.get("report"):
        bad.append("report differs from the one re-derived from the events")
    return bad


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="sdcguard assignment")
    sub = ap.add_subparsers(dest="cmd", required=True)
    i = sub.add_parser("inspect")
    i.add_argument("events")
    i.add_argument("--json", action="store_true")
    k = sub.add_parser("packet")
    k.add_argument("events")
    k.add_argument("--out", required=True)
    v = sub.add_parser("verify")
    v.add_argument("packet")
    a = ap.parse_args(argv)
    try:
        if a.cmd == "verify":
            with open(a.packet) as f:
                bad = verify_packet(json.load(f))
            print("packet verified" if not bad else "FAIL " + "; ".join(bad))
            return 0 if not bad else 1
        ev = parse_records(a.events)
    except (OSError, ValueError) as e:
        print(f"assignment: {e}", file=sys.stderr)
        return 2
    if a.cmd == "packet":
        p = create_packet(ev)
        with open(a.out, "w") as f:
            json.dump(p, f, sort_keys=True)
        print(render_report(p["report"]))
        return 0
    r = inspect_payload(ev)
    print(json.dumps(r, indent=1) if a.json else render_report(r))
    return {"PASS": 0, "HOLD": 1, "FAIL": 3}[r["verdict"]]


if __name__ == "__main__":
    raise SystemExit(main())
