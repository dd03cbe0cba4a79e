"""The saved regression case of this package, exported and judged offline: the prefill/decode abort that frees a
KV block while the aborted request's write is in flight (a stale write into the next request's block).

    python -m sdcguard_b200.evidence.regression run [--variant buggy|fixed] [--json]   # re-run the harness, judge
    python -m sdcguard_b200.evidence.regression export OUT_DIR                           # portable case bundle
    python -m sdcguard_b200.evidence.regression verify OUT_DIR                           # check it, run nothing
    sdcguard regression ...

The case (`evidence/data/pd_abort_case.json`) pins the condition, the harness (the lifetime protocol model
"pd-abort" under the delay-bounded explorer, budget 2) and, per variant, the rules the harness must report and the
SHA-256 of its canonical result. `judge` passes a result when its digest is the saved one and its rules are the
expected ones (buggy: R2, a read of a reallocated block; fixed: none); a different digest with the expected rules
is "changed" (the harness's exploration moved, the verdict did not), anything else fails. The bundle holds the case,
both saved results and a manifest of digests; verifying it executes none of its files.

Reference: src/sdcguard/regression.py:1-10 (`historical_case`, `judge`, `export_case`, `run_export`),
case_bundle.py:1-5 (`payloads`, `export_bundle`, `verify_bundle`: portable pinned files, verified without executing).
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os

CASE_FILE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "data", "pd_abort_case.json")


def digest(value) -> str:
    return hashlib.sha256(json.dumps(value, sort_keys=True, separators=(",", ":")).encode()).hexdigest()


def historical_case() -> dict:
    with open(CASE_FILE) as f:
        return json.load(f)


def run_case(variant: str) -> dict:
    from ..lifetime.explore import explore
    from ..lifetime.models import make
    h = historical_case()["harness"]
    return explore(make(f"{h['model']}:{variant}"), h["budget"], max_steps=h["max_steps"]).as_dict()


def judge(result: dict, variant: str) -> dict:
    case = historical_case()
    out = {"case": case["case"], "variant": variant, "status": "fail", "why": []}
    if variant not in case["expected"] or not isinstance(result, dict):
        out["why"].append("unknown variant or malformed result")
        return out
    exp = case["expected"][variant]
    rules = sorted({f.get("rule") for f in result.get("findings", [])})
    same_rules = rules == sorted(exp["rules"])
    d = digest(result)
    if same_rules and d == exp["result_sha256"]:
        out["status"] = "pass"
    elif same_rules:
        out["status"] = "changed"
        out["why"].append("same rules, different exploration (digest differs)")
    else:
        out["why"].append(f"rules {rules} where {exp['rules']} were expected")
    out["result_sha256"] = d
    return out


def payloads() -> dict:
    case = historical_case()
    return {"CASE.json": case, "RESULT_buggy.json": run_case("buggy"), "RESULT_fixed.json": run_case("fixed")}


def export_case(out: str) -> dict:
    os.makedirs(out, exist_ok=True)
    man = {"schema": "sdcguard_b200.case-bundle.v1", "files": {}}
    for name, doc in payloads().items():
        raw = json.dumps(doc, sort_keys=True, indent=1).encode()
        with open(os.path.join(out, name), "wb") as f:
            f.write(raw)
        man["files"][name] = hashlib.sha256(raw).hexdigest()
    with open(os.path.join(out, "MANIFEST.json"), "w") as f:
        json.dump(man, f, indent=1, sort_keys=True)
    return man


def verify_bundle(out: str) -> list[str]:
    bad = []
    try:
        with open(os.path.join(out, "MANIFEST.json")) as f:
            man = json.load(f)
    except (OSError, ValueError) as e:
        return [f"manifest unreadable: {e}"]
    if set(os.listdir(out)) - set(man["files"]) - {"MANIFEST.json"}:
        bad.append("files not in the manifest")
    docs = {}
    for name, sha in man["files"].items():
        try:
            with open(os.path.join(out, name), "rb") as f:
                raw = f.read()
        except OSError:
            bad.append(f"{name}: missing")
            continue
        if hashlib.sha256(raw).hexdigest() != sha:
            bad.append(f"{name}: digest differs")
        docs[name] = json.loads(raw)
    case = docs.get("CASE.json")
    if case is not None and digest(case) != digest(historical_case()):
        bad.append("CASE.json differs from this package's saved case")
    for v in ("buggy", "fixed"):
        r = docs.get(f"RESULT_{v}.json")
        if r is not None and judge(r, v)["status"] != "pass":
            bad.append(f"RESULT_{v}.json does not reproduce the saved result")
    return bad


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="sdcguard regression")
    sub = ap.add_subparsers(dest="cmd", required=True)
    r = sub.add_parser("run")
    r.add_argument("--variant", choices=("buggy", "fixed"))
    r.add_argument("--json", action="store_true")
    e = sub.add_parser("export")
    e.add_argument("out")
    v = sub.add_parser("verify")
    v.add_argument("out")
    a = ap.parse_args(argv)
    if a.cmd == "export":
        m = export_case(a.out)
        print(f"exported {len(m['files'])} files to {a.out}")
        return 0
    if a.cmd == "verify":
        bad = verify_bundle(a.out)
        print("case bundle verified" if not bad else "\n".join("FAIL " + b for b in bad))
        return 0 if not bad else 1
    res = [judge(run_case(v), v) for v in ([a.variant] if a.variant else ["buggy", "fixed"])]
    for j in res:
        print(json.dumps(j) if a.json else f"{j['variant']}: {j['status']}" + (f" ({'; '.join(j['why'])})"
                                                                              if j["why"] else ""))
    return 0 if all(j["status"] == "pass" for j in res) else 1


if __name__ == "__main__":
    raise SystemExit(main())
