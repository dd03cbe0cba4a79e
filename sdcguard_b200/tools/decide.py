"""One decision on one proposed serving-stack change, with its questions kept apart.

    python -m sdcguard_b200.tools.decide --baseline qual/baseline.json --candidate qual/candidate.json \\
        [--policy policy.json] [--kernels before.json after.json] [--alerts alerts.jsonl] --out decision.json
    python -m sdcguard_b200.tools.decide --applies decision.json --url http://127.0.0.1:8000

Sections (each judged on its own evidence, never by comparing the candidate's numbers with the baseline's):

  arithmetic    FAULT (the candidate's checks alarmed, or an alert in --alerts) / NO FAULT OBSERVED (its checks ran:
                checks went up under load and every checked op ran) / INCONCLUSIVE (no evidence that checks ran)
  protection    PROTECTED / NOT PROTECTED: `ready` on the candidate
  isolation     NO LEAK SEEN / LEAK / INCONCLUSIVE: a request's greedy output does not depend on the request
                before it or on its batch
  consistency   CONSISTENT / INCONSISTENT: decoded tokens equal the prefilled prediction of the same context
  performance   OK / REGRESSED: candidate throughput at least policy min_throughput_ratio (default 0.9) of baseline
  kernels       (with --kernels) the library kernels the change added, and whether any matches a listed issue

decision: ACCEPT when arithmetic is NO FAULT OBSERVED and every other section passes (or is waived by the policy's
`waive` list); REJECT on a FAULT or a failed section; INCONCLUSIVE otherwise. The accepted candidate's stack record is
kept, so `ready --qualified decision.json` can tell later whether a server still runs that stack (`--applies` does
the same from here).

Reference: src/sdcguard/decide.py:1-30 (sections and verdict words), `arithmetic` :274.
"""
from __future__ import annotations

import argparse
import json
import time
from typing import Optional

from . import _client

DEFAULT_POLICY = {"min_throughput_ratio": 0.9, "waive": []}


def _arith(cand: dict, alerts: list) -> dict:
    m = _client.parse_metrics(cand.get("metrics", ""))
    if alerts or m.get("sdcguard_alarms_total", 0) > 0:
        return {"verdict": "FAULT", "why": [f"{int(m.get('sdcguard_alarms_total', 0))} alarms, {len(alerts)} alerts"]}
    ran = m.get("sdcguard_checks_total", 0) > 0 and m.get("sdcguard_ops_checked", 0) == m.get("sdcguard_ops_total", -1)
    if not ran or m.get("sdcguard_protected", 0) != 1:
        return {"verdict": "INCONCLUSIVE", "why": ["no evidence that the candidate's checks ran"]}
    return {"verdict": "NO FAULT OBSERVED", "checks": int(m["sdcguard_checks_total"]),
            "ops_checked": int(m["sdcguard_ops_checked"])}


def decide(base: dict, cand: dict, policy: Optional[dict] = None, alerts: Optional[list] = None,
           kernels: Optional[tuple] = None) -> dict:
    pol = {**DEFAULT_POLICY, **(policy or {})}
    sec = {"arithmetic": _arith(cand, alerts or [])}
    r = cand["ready"]["verdict"]
    sec["protection"] = {"verdict": "PROTECTED" if r == "PROTECTED" else "NOT PROTECTED", "ready": r}
    iso = cand["isolation"]
    sec["isolation"] = {"verdict": iso["verdict"],
                        "failed": sum(1 for r in iso.get("probes", []) if r.get("verdict") != "NO LEAK SEEN")}
    sec["consistency"] = {"verdict": cand["consistency"]["verdict"], "checks": cand["consistency"]["checks"]}
    b, c = base["perf"]["total_tokens_per_s"], cand["perf"]["total_tokens_per_s"]
    ratio = c / b if b else 0.0
    sec["performance"] = {"verdict": "OK" if ratio >= pol["min_throughput_ratio"] and not cand["perf"]["errors"]
                          else "REGRESSED", "throughput_ratio": round(ratio, 4), "baseline": b, "candidate": c}
    if kernels:
        from .kernels import diff
        d = diff(*kernels)
        flagged = [k for k in d["only_after"] if kernels[1]["kernels"][k]["flags"]]
        sec["kernels"] = {"verdict": "FLAGGED" if flagged else "OK", "added": d["only_after"], "flagged": flagged}
    passing = {"arithmetic": "NO FAULT OBSERVED", "protection": "PROTECTED", "isolation": "NO LEAK SEEN",
               "consistency": "CONSISTENT", "performance": "OK", "kernels": "OK"}
    failed = [k for k, v in sec.items() if v["verdict"] != passing[k] and k not in pol["waive"]]
    if sec["arithmetic"]["verdict"] == "FAULT":
        decision = "REJECT"
    elif sec["arithmetic"]["verdict"] == "INCONCLUSIVE":
        decision = "INCONCLUSIVE"
    else:
        decision = "REJECT" if failed else "ACCEPT"
    return {"format": "sdcguard-b200-decision/1", "time": time.time(), "decision": decision, "failed": failed,
            "sections": sec, "policy": pol, "baseline_stack": base.get("stack"), "candidate_stack": cand.get("stack")}


def applies(decision: dict, url: str) -> dict:
    from .ready import qualified
    m = _client.scrape(url)
    if m is None:
        return {"applies": False, "why": ["no metrics"]}
    q = qualified(m, decision)
    return {"applies": q is None, "why": [] if q is None else q["why"]}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m sdcguard_b200.tools.decide")
    ap.add_argument("--baseline")
    ap.add_argument("--candidate")
    ap.add_argument("--policy")
    ap.add_argument("--alerts")
    ap.add_argument("--kernels", nargs=2)
    ap.add_argument("--out")
    ap.add_argument("--applies")
    ap.add_argument("--url")
    a = ap.parse_args(argv)

    def load(p):
        with open(p) as f:
            return json.load(f)

    if a.applies:
        r = applies(load(a.applies), a.url)
        print(json.dumps(r))
        return 0 if r["applies"] else 1
    alerts = []
    if a.alerts:
        with open(a.alerts) as f:
            alerts = [json.loads(x) for x in f if x.strip()]
    d = decide(load(a.baseline), load(a.candidate), load(a.policy) if a.policy else None, alerts,
               (load(a.kernels[0]), load(a.kernels[1])) if a.kernels else None)
    if a.out:
        with open(a.out, "w") as f:
            json.dump(d, f, indent=1)
    print(json.dumps({"decision": d["decision"], "failed": d["failed"]}))
    return {"ACCEPT": 0, "REJECT": 1}.get(d["decision"], 2)


if __name__ == "__main__":
    raise SystemExit(main())
