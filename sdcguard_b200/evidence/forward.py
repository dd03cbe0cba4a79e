"""Inspection of the recorded forward inputs of a run of this engine: for every forward pass of a request, was every
KV page in its block table that request's own page (or a prefix page shared with it), of the live generation?

    python -m sdcguard_b200.evidence.forward inspect lifetime.jsonl [--json]
    python -m sdcguard_b200.evidence.forward packet lifetime.jsonl --out PACKET.json
    python -m sdcguard_b200.evidence.forward verify PACKET.json
    sdcguard forward-inputs ...

The engine records each forward pass as a "forward" event in the lifetime stream (`EventSink.forward`: phase,
request, the block table's [pool, page, generation] entries, first and last position). Ownership is replayed from
the same stream (`evidence.assignment.Ownership`), so each forward event is judged against the state at that point.
Findings per forward entry: a page that is not live, a live page of another generation (a stale table entry), a page
owned by another request and not shared with this one; and a block table shorter than its positions need. It performs
no device work and infers no ownership the events do not record.

Reference: src/sdcguard/forward_report.py:1-10 (`parse_records`, `inspect_payload`, `render_report`,
`create_packet`, `verify_packet`).
"""
from __future__ import annotations

import argparse
import hashlib
import json
import sys

from . import catalog
from .assignment import Ownership, parse_records

SCHEMA = "sdcguard_b200.forward-packet.v1"
PAGE_TOKENS = 16


def inspect_payload(events: list[dict], page_tokens: int = PAGE_TOKENS) -> dict:
    own = Ownership()
    issues, passes = [], 0
    for i, e in enumerate(events):
        if e["ev"] != "forward":
            own.apply(i, e)
            continue
        passes += 1
        req = e["request"]
        regs = e.get("regions", [])
        first, last = e.get("positions", [0, -1])
        if last >= first and len(regs) * page_tokens <= last:
            issues.append({"event": i, "kind": "table_too_short", "request": req, "pages": len(regs),
                           "last_position": last})
        for pool, idx, gen in regs:
            h = own.holders((pool, idx))
            if h is None:
                issues.append({"event": i, "kind": "page_not_live", "request": req, "region": [pool, idx]})
            elif h[1] != gen:
                issues.append({"event": i, "kind": "stale_generation", "request": req, "region": [pool, idx],
                               "gen": gen, "live_gen": h[1]})
            elif h[0] != req and req not in h[2]:
                issues.append({"event": i, "kind": "foreign_page", "request": req, "region": [pool, idx],
                               "owner": h[0]})
    if not passes:
        f = catalog.finding("forward.owned_pages", "unknown", "the events record no forward pass",
                            "recorded lifetime events")
    else:
        f = catalog.finding("forward.owned_pages", "violated" if issues else "satisfied",
                            f"{len(issues)} block-table entr(ies) outside the request's pages" if issues else
                            f"all {passes} forward passes read only their requests' pages",
                            "recorded forward inputs and ownership", {"forward_passes": passes})
    return {"schema": "sdcguard_b200.forward-report.v1", "forward_passes": passes, "issues": issues,
            "findings": [f], "verdict": "FAIL" if issues else ("PASS" if passes else "HOLD"),
            "scope": "recorded forward inputs of one run against recorded ownership"}


def render_report(r: dict) -> str:
    lines = [f"forward inputs: {r['verdict']} ({r['forward_passes']} forward passes)"]
    lines += [f"  {x['kind']} at event {x['event']}: request {x['request']}" +
              (f", region {x['region']}" if "region" in x else "") for x in r["issues"][:50]]
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
    ap = argparse.ArgumentParser(prog="sdcguard forward-inputs")
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
        print(f"forward-inputs: {e}", file=sys.stderr)
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
