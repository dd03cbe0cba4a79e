"""One envelope for several evidence sections (deployment contracts, recording assessment, client inventory,
overhead, assignment, forward inputs), each kept in its own scope: combining sections never lets one section's
findings speak for another's.

    python -m sdcguard_b200.evidence.report build OUT.json --section config=cfg.json --section inventory=inv.json
    python -m sdcguard_b200.evidence.report verify OUT.json            # sdcguard report-verify OUT.json
    python -m sdcguard_b200.evidence.report render OUT.json

A section file is the JSON an evaluator wrote (`config-safety --json`, `assess --json`, `inventory --json`, ...).
`build` extracts its findings (every object with the finding shape, wherever it sits), keys each one by
(section, worker or subject, rule id), and records the section's canonical digest and the catalog digest. `verify`
recomputes every digest, re-checks every finding against the catalog and fails on any difference; it re-runs no
evaluator (re-evaluation is each section's own tool).

Reference: src/sdcguard/evidence_report.py:1-10 (`build`, `render`, `finding_key`, `catalog_hash`,
`static_findings`), evidence_envelope.py (bounded versioned envelope), evidence_entry.py (routing).
"""
from __future__ import annotations

import argparse
import hashlib
import json
import sys

from . import catalog

SCHEMA = "sdcguard_b200.evidence-report.v1"
MAX_SECTION_BYTES = 16 << 20


def _canon(v) -> bytes:
    return json.dumps(v, sort_keys=True, separators=(",", ":"), allow_nan=False).encode()


def _sha(v) -> str:
    return hashlib.sha256(_canon(v)).hexdigest()


def findings_of(doc, subject: str = "") -> list[tuple[str, dict]]:
    """(subject, finding) pairs: every finding-shaped object in doc; the subject is the id of the nearest enclosing
    object that has one (a worker), else ''."""
    out = []
    if isinstance(doc, dict):
        if not catalog.validate_finding(doc):
            return [(subject, doc)]
        sub = doc.get("id") if isinstance(doc.get("id"), str) and "rules" in doc else subject
        for v in doc.values():
            out += findings_of(v, sub)
    elif isinstance(doc, list):
        for v in doc:
            out += findings_of(v, subject)
    return out


def finding_key(section: str, subject: str, f: dict) -> str:
    return f"{section}/{subject}/{f['id']}" if subject else f"{section}/{f['id']}"


def build(sections: dict) -> dict:
    secs, allf = {}, {}
    for name, doc in sorted(sections.items()):
        fs = findings_of(doc)
        keys = []
        for subj, f in fs:
            k = finding_key(name, subj, f)
            if k in allf:
                raise ValueError(f"duplicate finding key {k}")
            allf[k] = f
            keys.append(k)
        secs[name] = {"sha256": _sha(doc), "verdict": doc.get("verdict") if isinstance(doc, dict) else None,
                      "scope": doc.get("scope") if isinstance(doc, dict) else None, "findings": sorted(keys),
                      "document": doc}     # sorted: a document's key order does not survive every JSON writer
    counts = {v: sum(1 for f in allf.values() if f["verdict"] == v) for v in catalog.VERDICTS}
    return {"schema": SCHEMA, "catalog_sha256": catalog.catalog_hash(), "sections": secs, "findings": allf,
            "counts": counts, "envelope_sha256": _sha({"sections": {k: v["sha256"] for k, v in secs.items()},
                                                       "findings": allf})}


def verify(env: dict) -> list[str]:
    """Problems with an envelope (empty: every digest and finding checks out)."""
    bad = []
    if env.get("schema") != SCHEMA:
        return [f"not a {SCHEMA} envelope"]
    if env.get("catalog_sha256") != catalog.catalog_hash():
        bad.append("built against another rule catalog")
    try:
        again = build({k: v["document"] for k, v in env["sections"].items()})
    except (KeyError, TypeError, ValueError) as e:
        return bad + [f"sections unreadable: {e}"]
    for k, v in env["sections"].items():
        if v.get("sha256") != again["sections"][k]["sha256"]:
            bad.append(f"section {k}: digest differs from its document")
        if v.get("findings") != again["sections"][k]["findings"]:
            bad.append(f"section {k}: finding list differs from its document")
    if env.get("findings") != again["findings"]:
        bad.append("findings differ from the sections' documents")
    for k, f in env.get("findings", {}).items():
        for p in catalog.validate_finding(f):
            bad.append(f"{k}: {p}")
    if env.get("envelope_sha256") != again["envelope_sha256"]:
        bad.append("envelope digest differs")
    return bad


def render(env: dict) -> str:
    lines = [f"evidence report ({len(env['sections'])} sections, catalog {env['catalog_sha256'][:12]})"]
    for name, s in env["sections"].items():
        lines.append(f"[{name}] verdict={s['verdict']} sha256={s['sha256'][:16]}")
        if s.get("scope"):
            lines.append(f"  scope: {s['scope']}")
        for k in s["findings"]:
            f = env["findings"][k]
            lines.append(f"  {f['verdict']:<15} {k}: {f['message']}")
    lines.append("counts: " + ", ".join(f"{k}={v}" for k, v in env["counts"].items()))
    return "\n".join(lines)


def _load(path: str):
    with open(path, "rb") as f:
        raw = f.read(MAX_SECTION_BYTES + 1)
    if len(raw) > MAX_SECTION_BYTES:
        raise ValueError(f"{path}: larger than {MAX_SECTION_BYTES} bytes")
    return json.loads(raw)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="sdcguard evidence")
    sub = ap.add_subparsers(dest="cmd", required=True)
    b = sub.add_parser("build")
    b.add_argument("out")
    b.add_argument("--section", action="append", default=[], help="NAME=FILE.json")
    v = sub.add_parser("verify")
    v.add_argument("report")
    r = sub.add_parser("render")
    r.add_argument("report")
    a = ap.parse_args(argv)
    if a.cmd == "build":
        secs = {}
        for s in a.section:
            name, _, path = s.partition("=")
            if not name or not path:
                print(f"evidence: bad --section {s!r}", file=sys.stderr)
                return 2
            secs[name] = _load(path)
        env = build(secs)
        with open(a.out, "w") as f:
            json.dump(env, f, indent=1, sort_keys=True)
        print(render(env))
        return 0
    env = _load(a.report)
    if a.cmd == "render":
        print(render(env))
        return 0
    bad = verify(env)
    for p in bad:
        print(f"FAIL {p}")
    print("report verified" if not bad else f"{len(bad)} problem(s)")
    return 0 if not bad else 1


def verify_main(argv=None) -> int:
    return main(["verify", *(argv or sys.argv[1:])])


if __name__ == "__main__":
    raise SystemExit(main())
