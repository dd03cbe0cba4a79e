"""Reconcile a declared client batch with a recording of this engine, offline: does every request the client sent
have exactly one recorded KV transfer, and is every recorded transfer one the client declared?

    python -m sdcguard_b200.evidence.inventory CLIENT.json RECORDING_DIR [--json]
    sdcguard inventory CLIENT.json RECORDING_DIR

CLIENT.json ("sdcguard_b200.client-inventory.v1"): {"workload": str, "requests": [{"client_request_id": str,
"prompt_sha256": hex, "prompt_tokens": int}]}; `prompt_sha256` is the SHA-256 of the prompt's token ids in the
recordings' canonical JSON encoding (`coverage.evidence.json_bytes`), as REQUEST_PLAN.json stores them
(`from_prompts` builds the file from token lists).

The join key is (prompt_sha256, prompt_tokens): a declared request matches when exactly one planned request of the
recording has that key, that request id is unique, and the recording's observer holds transfer records for it.
Anything else (no match, two matches, a duplicate declaration, a transfer no declared request explains) leaves the
status "unknown" with the reason; "complete" only when every declared request matched and nothing is left over.
An exact join establishes recorded coverage of the declared batch, not of all server traffic and not isolation.

Reference: src/sdcguard/client_inventory.py:1-10 (`reconcile`: unknown for any absent, malformed, extra or ambiguous
attempt), `validate_inventory`, `from_performance`.
"""
from __future__ import annotations

import argparse
import json
import os
from collections import Counter, defaultdict

from . import catalog

SCHEMA = "sdcguard_b200.client-inventory.v1"
MAX_REQUESTS = 1_000_000
SCOPE = "declared client batch against one recording; not all server traffic, identities or request isolation"


def from_prompts(prompts: dict, workload: str = "declared-batch") -> dict:
    """{client_request_id: token id list} -> an inventory document."""
    from ..coverage import evidence as ev
    return {"schema": SCHEMA, "workload": workload,
            "requests": [{"client_request_id": cid, "prompt_sha256": ev.digest(ev.json_bytes([int(x) for x in t])),
                          "prompt_tokens": len(t)} for cid, t in prompts.items()]}


def validate_inventory(doc) -> list[dict]:
    if not isinstance(doc, dict) or doc.get("schema") != SCHEMA:
        raise ValueError(f"not a {SCHEMA} document")
    rows = doc.get("requests")
    if not isinstance(rows, list) or len(rows) > MAX_REQUESTS:
        raise ValueError("requests must be a bounded list")
    for i, r in enumerate(rows):
        if (not isinstance(r, dict) or not isinstance(r.get("client_request_id"), str)
                or not isinstance(r.get("prompt_sha256"), str) or len(r["prompt_sha256"]) != 64
                or type(r.get("prompt_tokens")) is not int or r["prompt_tokens"] < 0):
            raise ValueError(f"malformed request at index {i}")
    return rows


def _load(path: str):
    with open(path, "rb") as f:
        return json.loads(f.read(64 << 20))


def reconcile(inventory: dict, recording: str) -> dict:
    res = {"schema": "sdcguard_b200.request-coverage.v1", "status": "unknown", "scope": SCOPE,
           "declared_requests": None, "matched_requests": 0, "recorded_requests": 0, "requests": [],
           "unexpected": [], "issues": []}
    try:
        rows = validate_inventory(inventory)
    except ValueError as e:
        res["issues"].append(str(e))
        return _finish(res)
    res["declared_requests"] = len(rows)
    try:
        plan = _load(os.path.join(recording, "REQUEST_PLAN.json"))
        observer = _load(os.path.join(recording, "OBSERVER.json"))
    except (OSError, ValueError) as e:
        res["issues"].append(f"recording unreadable: {e}")
        return _finish(res)
    planned = plan.get("requests", []) if isinstance(plan, dict) else []
    res["recorded_requests"] = len(planned)
    by_key = defaultdict(list)
    rid_count = Counter()
    for p in planned:
        if isinstance(p, dict):
            by_key[(p.get("prompt_sha256"), p.get("prompt_tokens"))].append(p.get("request_id"))
            rid_count[p.get("request_id")] += 1
    transferred = Counter(r.get("request_id") for r in observer.get("records", []) if isinstance(r, dict))
    ids = Counter(r["client_request_id"] for r in rows)
    keys = Counter((r["prompt_sha256"], r["prompt_tokens"]) for r in rows)
    used = set()
    for r in rows:
        k = (r["prompt_sha256"], r["prompt_tokens"])
        m = by_key.get(k, [])
        reason = None
        if ids[r["client_request_id"]] != 1:
            reason = "duplicate client request id"
        elif keys[k] != 1:
            reason = "two declared requests share a prompt (no unique join)"
        elif not m:
            reason = "no planned request with this prompt"
        elif len(m) != 1:
            reason = "several planned requests have this prompt"
        elif rid_count[m[0]] != 1:
            reason = "recorded request id is not unique"
        elif not transferred.get(m[0]):
            reason = "planned, but no transfer record"
        res["requests"].append({"client_request_id": r["client_request_id"],
                                "engine_request": m[0] if len(m) == 1 else None,
                                "status": "unknown" if reason else "matched",
                                "reason": reason or "unique prompt match with transfer records"})
        used.update(m)
        if reason is None:
            res["matched_requests"] += 1
    for rid in transferred:
        if rid not in used:
            res["unexpected"].append({"request": rid, "reason": "transfer outside the declared batch"})
    if any(q["status"] != "matched" for q in res["requests"]):
        res["issues"].append("not every declared request has one unambiguous recorded transfer")
    if res["unexpected"]:
        res["issues"].append("the recording holds transfers the declared batch does not explain")
    if not res["issues"]:
        res["status"] = "complete"
    return _finish(res)


def _finish(res: dict) -> dict:
    res["findings"] = [catalog.finding("inventory.complete", "satisfied" if res["status"] == "complete" else "unknown",
                                       f"{res['matched_requests']} of {res['declared_requests']} declared requests "
                                       f"matched" + (f"; {res['issues'][0]}" if res["issues"] else ""),
                                       "client inventory joined with the recording",
                                       {"unexpected": len(res["unexpected"])})]
    res["verdict"] = "PASS" if res["status"] == "complete" else "HOLD"
    return res


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="sdcguard inventory")
    ap.add_argument("inventory")
    ap.add_argument("recording")
    ap.add_argument("--json", action="store_true")
    a = ap.parse_args(argv)
    r = reconcile(_load(a.inventory), a.recording)
    if a.json:
        print(json.dumps(r, indent=1))
    else:
        print(f"{r['status']}: {r['matched_requests']}/{r['declared_requests']} matched, "
              f"{len(r['unexpected'])} unexpected")
        for i in r["issues"]:
            print(f"  {i}")
    return 0 if r["status"] == "complete" else 1


if __name__ == "__main__":
    raise SystemExit(main())
