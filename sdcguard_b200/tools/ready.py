"""Is this server's math being checked right now? Asked from outside, from its metrics.

    python -m sdcguard_b200.tools.ready http://127.0.0.1:8000 [--probe] [--max-z 6] [--qualified decision.json]

Reads /metrics twice, a few seconds apart (with --probe: sends two short requests in between) and answers:

  PROTECTED          metrics present, sdcguard_protected 1, every checked op has run checks, the alarm line is at most
                     --max-z, results have been read back, the worker did not restart, and the checks went up while
                     tokens were produced
  IDLE               all of that holds but no tokens were produced between the reads (use --probe for a definite
                     answer)
  NOT PROTECTED      no metrics, protected 0, ops never checked, an alarm line above --max-z, or tokens produced while
                     the checks did not move
  FAULT FOUND        the alarm counter is above zero: take the server out of rotation and screen the GPU
  NOT THE QUALIFIED STACK / NOT QUALIFIED   with --qualified: the server's stack record differs from the one the
                     decision accepted, or the decision did not accept

Exit code 0 for PROTECTED (and IDLE), 1 otherwise.

Reference: src/sdcguard/ready.py:1-40 (the conditions and verdict words), `scrape` :109, `qualified` :245.
"""
from __future__ import annotations

import argparse
import json
import time
from typing import Callable, Optional

from . import _client


def _stack(m: dict) -> dict:
    rows = m.get("sdcguard_stack_info{}") or []
    return rows[0][0] if rows else {}


def _worker(m: dict) -> dict:
    rows = m.get("sdcguard_worker_info{}") or []
    return rows[0][0] if rows else {}


def judge(m1: Optional[dict], m2: Optional[dict], max_z: float = 6.0) -> dict:
    """The verdict from two scrapes (pure function of the metrics)."""
    if m1 is None or m2 is None:
        return {"verdict": "NOT PROTECTED", "why": ["no metrics (server down, or not this library's server)"]}
    why = []
    if m2.get("sdcguard_alarms_total", 0) > 0:
        return {"verdict": "FAULT FOUND", "why": [f"{int(m2['sdcguard_alarms_total'])} alarms"]}
    if m2.get("sdcguard_protected", 0) != 1:
        why.append("checks are off (sdcguard_protected 0)")
    if m2.get("sdcguard_alarm_line", 1e9) > max_z:
        why.append(f"alarm line {m2.get('sdcguard_alarm_line')} above {max_z}")
    if _worker(m1).get("started") != _worker(m2).get("started") or _worker(m1).get("pid") != _worker(m2).get("pid"):
        why.append("the worker restarted between the reads")
    ops, checked = m2.get("sdcguard_ops_total", 0), m2.get("sdcguard_ops_checked", 0)
    tokens = m2.get("sdcguard_generated_tokens_total", 0) - m1.get("sdcguard_generated_tokens_total", 0)
    checks = m2.get("sdcguard_checks_total", 0) - m1.get("sdcguard_checks_total", 0)
    if why:
        return {"verdict": "NOT PROTECTED", "why": why}
    if m2.get("sdcguard_polls_total", 0) < 1 or ops == 0:
        return {"verdict": "IDLE", "why": ["no check has run yet (send a request, or use --probe)"]}
    if checked < ops:
        return {"verdict": "NOT PROTECTED", "why": [f"{int(ops - checked)} of {int(ops)} checked ops never ran"]}
    if tokens > 0 and checks <= 0:
        return {"verdict": "NOT PROTECTED", "why": ["tokens were produced while the checks did not move"]}
    if tokens <= 0:
        return {"verdict": "IDLE", "why": ["no tokens between the reads"]}
    return {"verdict": "PROTECTED", "why": [], "checks_between_reads": checks, "tokens_between_reads": tokens}


def qualified(m: dict, decision: dict) -> Optional[dict]:
    if decision.get("decision") != "ACCEPT":
        return {"verdict": "NOT QUALIFIED", "why": [f"the decision was {decision.get('decision')}"]}
    want = decision.get("candidate_stack") or {}
    got = _stack(m)
    diff = {k: (want.get(k), got.get(k)) for k in set(want) | set(got) if want.get(k) != got.get(k)}
    if diff:
        return {"verdict": "NOT THE QUALIFIED STACK", "why": [f"{k}: qualified {a}, serving {b}"
                                                              for k, (a, b) in sorted(diff.items())]}
    return None


def check(base: str, probe: bool = False, wait: float = 2.0, max_z: float = 6.0,
          decision: Optional[dict] = None, scrape: Callable = _client.scrape,
          complete: Callable = _client.complete) -> dict:
    m1 = scrape(base)
    if probe and m1 is not None:
        for i in range(2):
            complete(base, [1 + i, 2, 3, 4], 4)
    else:
        time.sleep(wait)
    m2 = scrape(base)
    r = judge(m1, m2, max_z)
    if decision is not None and m2 is not None and r["verdict"] in ("PROTECTED", "IDLE"):
        q = qualified(m2, decision)
        if q:
            r = q
    r["stack"] = _stack(m2 or {})
    return r


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m sdcguard_b200.tools.ready")
    ap.add_argument("url")
    ap.add_argument("--probe", action="store_true")
    ap.add_argument("--wait", type=float, default=2.0)
    ap.add_argument("--max-z", type=float, default=6.0)
    ap.add_argument("--qualified")
    a = ap.parse_args(argv)
    dec = None
    if a.qualified:
        with open(a.qualified) as f:
            dec = json.load(f)
    r = check(a.url, a.probe, a.wait, a.max_z, dec)
    print(json.dumps(r))
    return 0 if r["verdict"] in ("PROTECTED", "IDLE") else 1


if __name__ == "__main__":
    raise SystemExit(main())
