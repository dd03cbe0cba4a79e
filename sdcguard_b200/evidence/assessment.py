"""Scoped, read-only assessment of one recorded prefill/decode run of this engine.

    python -m sdcguard_b200.evidence.assessment RECORDING_DIR --events lifetime.jsonl [--ready-url URL] [--json]

It combines, without running anything that changes state:

  coverage     the KV-checksum coverage gate of the recording (`coverage.own`): PASS when every request's transferred
               KV was compared in full, HOLD otherwise (e.g. cached prefix pages reused without re-verification)
  lifetime     the recorded page-lifetime events replayed through the ledger (`lifetime.adapter`): no rule broken
  readiness    optional: `tools.ready` against the serving endpoint (read-only metrics)

verdict: PASS when coverage passed, no lifetime rule was broken and (when asked) the server is PROTECTED; FAIL when a
lifetime rule was broken, a checksum mismatched or readiness found a fault; HOLD otherwise. The scope line says what
this does not cover: it is about this recording, not a guarantee about the server's later traffic.

Reference: src/sdcguard/assessment.py:1-20 (scope, read-only combination; `assess` :114).
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
from typing import Optional

SCOPE = ("this recording's KV transfers and page lifetimes on this engine; no guarantee about other traffic, other "
         "engines or the arithmetic outside the recorded checks")


def _sha(path: str) -> Optional[str]:
    try:
        with open(path, "rb") as f:
            return hashlib.sha256(f.read()).hexdigest()
    except OSError:
        return None


def assess(recording: str, events: Optional[str] = None, ready_url: Optional[str] = None) -> dict:
    from ..coverage import own
    from ..lifetime import adapter
    out: dict = {"format": "sdcguard-b200-assessment/1", "scope": SCOPE, "recording": os.path.abspath(recording)}
    try:
        gate = own.inspect(recording)
        reasons = sorted({r for q in gate.get("requests", []) for r in q.get("reasons", [])})
        out["coverage"] = {"decision": gate.get("decision"), "hold_reasons": gate.get("hold_reasons", []),
                           "requests": len(gate.get("requests", [])), "reasons": reasons}
    except Exception as e:  # noqa: BLE001  (an unreadable recording is part of the answer)
        out["coverage"] = {"decision": "ERROR", "error": f"{type(e).__name__}: {e}"}
    if events:
        lt = adapter.check(adapter.load(events))
        out["lifetime"] = {"events": lt["events"], "violations": lt["violations"], "sha256": _sha(events)}
    else:
        out["lifetime"] = {"events": 0, "violations": [], "note": "no events recorded: not assessed"}
    if ready_url:
        from ..tools import ready
        out["readiness"] = ready.check(ready_url, probe=False)
    mismatch = any("mismatch" in r for r in out["coverage"].get("reasons", []))
    fault = out.get("readiness", {}).get("verdict") == "FAULT FOUND"
    if out["lifetime"]["violations"] or mismatch or fault:
        v = "FAIL"
    elif (out["coverage"].get("decision") == "PASS" and events
          and (not ready_url or out["readiness"]["verdict"] == "PROTECTED")):
        v = "PASS"
    else:
        v = "HOLD"
    out["verdict"] = v
    out["findings"] = _findings(out, bool(events), bool(ready_url))
    return out


def _findings(out: dict, have_events: bool, asked_ready: bool) -> list[dict]:
    """The assessment's parts as catalog findings (for `evidence.report`)."""
    from . import catalog
    cov = out["coverage"]
    d = cov.get("decision")
    fs = [catalog.finding("recording.coverage", {"PASS": "satisfied", "HOLD": "unknown"}.get(d, "violated")
                          if d != "ERROR" else "unknown",
                          f"coverage gate {d}" + (f": {', '.join(cov.get('hold_reasons', []))}"
                                                  if cov.get("hold_reasons") else ""),
                          "recording", {"requests": cov.get("requests"), "reasons": cov.get("reasons", [])})]
    lt = out["lifetime"]
    fs.append(catalog.finding("recording.lifetime", "unknown" if not have_events else
                              ("violated" if lt["violations"] else "satisfied"),
                              "no lifetime events recorded" if not have_events else
                              f"{len(lt['violations'])} ledger violation(s) in {lt['events']} events",
                              "recorded lifetime events", {"events": lt.get("events", 0)}))
    if asked_ready:
        rv = out["readiness"].get("verdict")
        fs.append(catalog.finding("recording.readiness", "satisfied" if rv == "PROTECTED" else
                                  ("violated" if rv == "FAULT FOUND" else "unknown"), f"readiness {rv}",
                                  "read-only endpoint"))
    return fs


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m sdcguard_b200.evidence.assessment")
    ap.add_argument("recording")
    ap.add_argument("--events")
    ap.add_argument("--ready-url")
    ap.add_argument("--json", action="store_true")
    a = ap.parse_args(argv)
    r = assess(a.recording, a.events, a.ready_url)
    if a.json:
        print(json.dumps(r, indent=1))
    else:
        print(f"{r['verdict']}: coverage {r['coverage'].get('decision')}, lifetime violations "
              f"{len(r['lifetime']['violations'])}" + (f", readiness {r['readiness']['verdict']}" if 'readiness' in r
                                                       else ""))
        print(f"scope: {r['scope']}")
    return {"PASS": 0, "HOLD": 2}.get(r["verdict"], 1)


if __name__ == "__main__":
    raise SystemExit(main())
