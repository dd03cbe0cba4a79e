"""Preservation policy for an engine upgrade: compare the evidence report of the running version (before) with the
report of the candidate (after), both built by `evidence.report` and verified first. The comparison approves nothing;
it says which established facts the candidate keeps.

    python -m sdcguard_b200.evidence.upgrade BEFORE.json AFTER.json [--json] [--out CMP.json]
    python -m sdcguard_b200.evidence.upgrade --verify CMP.json BEFORE.json AFTER.json
    sdcguard upgrade BEFORE.json AFTER.json

Per finding key (section / subject / rule):
  preserved   satisfied before and after (or not_applicable both times)
  regressed   satisfied before, violated after
  lost        satisfied before, unknown or absent after (a fact the candidate no longer establishes)
  improved    violated or unknown before, satisfied after
  new         absent before
  unchanged   any other pair with the same verdict
verdict: PRESERVED when nothing regressed or was lost, REGRESSED when something regressed, INCOMPLETE otherwise.
A comparison file carries both envelopes' digests; `--verify` recomputes it from the two reports.

Reference: src/sdcguard/upgrade.py:1-10 (`compare_packets`, `verify_comparison`), upgrade_policy.py:1-10 (pure
policy over already verified reports), upgrade_combined.py, upgrade_entry.py.
"""
from __future__ import annotations

import argparse
import json
import sys

from . import report

SCHEMA = "sdcguard_b200.upgrade-comparison.v1"
GOOD = ("satisfied", "not_applicable")


def classify(before, after) -> str:
    vb = before["verdict"] if before else None
    va = after["verdict"] if after else None
    if vb is None:
        return "new"
    if vb in GOOD:
        if va in GOOD:
            return "preserved"
        if va == "violated":
            return "regressed"
        return "lost"
    if va in GOOD:
        return "improved"
    return "unchanged"


def compare(before: dict, after: dict) -> dict:
    for name, env in (("before", before), ("after", after)):
        bad = report.verify(env)
        if bad:
            raise ValueError(f"{name} report does not verify: {bad[0]}")
    keys = sorted(set(before["findings"]) | set(after["findings"]))
    rows = []
    for k in keys:
        b, a = before["findings"].get(k), after["findings"].get(k)
        rows.append({"key": k, "before": b["verdict"] if b else None, "after": a["verdict"] if a else None,
                     "outcome": classify(b, a)})
    count = {o: sum(1 for r in rows if r["outcome"] == o)
             for o in ("preserved", "regressed", "lost", "improved", "new", "unchanged")}
    verdict = "REGRESSED" if count["regressed"] else ("INCOMPLETE" if count["lost"] else "PRESERVED")
    return {"schema": SCHEMA, "before_sha256": before["envelope_sha256"], "after_sha256": after["envelope_sha256"],
            "rows": rows, "counts": count, "verdict": verdict,
            "scope": "facts established by the two verified reports; no engine was run and nothing is approved"}


def verify_comparison(cmp: dict, before: dict, after: dict) -> list[str]:
    try:
        again = compare(before, after)
    except ValueError as e:
        return [str(e)]
    return [] if again == cmp else ["comparison differs from the one recomputed from the two reports"]


def render(c: dict) -> str:
    lines = [f"upgrade: {c['verdict']}  " + ", ".join(f"{k}={v}" for k, v in c["counts"].items())]
    lines += [f"  {r['outcome']:<10} {r['key']}: {r['before']} -> {r['after']}" for r in c["rows"]
              if r["outcome"] not in ("preserved", "unchanged")]
    return "\n".join(lines)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="sdcguard upgrade")
    ap.add_argument("before")
    ap.add_argument("after")
    ap.add_argument("--json", action="store_true")
    ap.add_argument("--out")
    ap.add_argument("--verify", metavar="CMP.json")
    a = ap.parse_args(argv)
    before, after = report._load(a.before), report._load(a.after)
    if a.verify:
        bad = verify_comparison(report._load(a.verify), before, after)
        print("comparison verified" if not bad else "FAIL " + bad[0])
        return 0 if not bad else 1
    try:
        c = compare(before, after)
    except ValueError as e:
        print(f"upgrade: {e}", file=sys.stderr)
        return 2
    if a.out:
        with open(a.out, "w") as f:
            json.dump(c, f, indent=1, sort_keys=True)
    print(json.dumps(c, indent=1) if a.json else render(c))
    return {"PRESERVED": 0, "INCOMPLETE": 1, "REGRESSED": 3}[c["verdict"]]


if __name__ == "__main__":
    raise SystemExit(main())
