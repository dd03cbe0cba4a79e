"""Overhead of the checks from matched runs, with the identity that makes two runs comparable.

    python -m sdcguard_b200.evidence.overhead prepare --config CFG.json --model-dir DIR --gpu-uuid GPU-... --out ID.json
    python -m sdcguard_b200.evidence.overhead compare ID.json --on on.jsonl --off off.jsonl [--bound 3] [--json]
    sdcguard overhead ...

prepare writes an identity document: the SHA-256 of the serving configuration, of the model directory's file
listing (`evidence.model_reference.capture`), the package version and the source digest of the installed package,
and the GPU UUID the operator names. compare reads two sets of bench lines (one JSON object per line, as `bench.py`
prints them; checked runs in --on, unchecked in --off) and reports the median throughput of each and the overhead
(1 - on / off) with its spread, after checking that every run names the same metric, config, GPU count and dtype,
and that the identity still describes this package. The GPU UUID and the on/off state are the operator's
declarations; a receipt is local consistency, not an attestation of the machine that ran.

Reference: src/sdcguard/overhead.py:1-10 (`summarize` of matched runs, offline preparation of their identity),
performance_identity.py:1-10 (`prepare_identity`, `validate_identity`, `measurement_digest`).
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import statistics
import sys
from typing import Optional

from . import catalog

SCHEMA = "sdcguard_b200.performance-identity.v1"


def _sha(v) -> str:
    return hashlib.sha256(json.dumps(v, sort_keys=True, separators=(",", ":")).encode()).hexdigest()


def package_digest() -> str:
    """SHA-256 over this package's Python and CUDA sources (names and bytes), in name order."""
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    h = hashlib.sha256()
    for d, dirs, files in sorted(os.walk(root)):
        dirs[:] = sorted(x for x in dirs if not x.startswith(("_", ".")))      # no build output, no caches
        for f in sorted(files):
            if f.endswith((".py", ".cu", ".cuh", ".h", ".cpp", ".json")):
                p = os.path.join(d, f)
                h.update(os.path.relpath(p, root).encode() + b"\0")
                with open(p, "rb") as fh:
                    h.update(hashlib.sha256(fh.read()).digest())
    return h.hexdigest()


def prepare_identity(config: dict, model_dir: Optional[str], gpu_uuid: str) -> dict:
    from .. import __version__
    from . import model_reference
    if not gpu_uuid.startswith("GPU-"):
        raise ValueError("gpu uuid must look like GPU-xxxxxxxx-...")
    model = model_reference.capture(model_dir) if model_dir else None
    doc = {"schema": SCHEMA, "config_sha256": _sha(config), "config": config,
           "model_capture_sha256": model["capture_sha256"] if model else None,
           "package_version": __version__, "package_sha256": package_digest(), "gpu_uuid": gpu_uuid}
    doc["identity_sha256"] = _sha({k: v for k, v in doc.items() if k != "identity_sha256"})
    return doc


def validate_identity(doc: dict) -> list[str]:
    bad = []
    if not isinstance(doc, dict) or doc.get("schema") != SCHEMA:
        return [f"not a {SCHEMA} document"]
    if doc.get("identity_sha256") != _sha({k: v for k, v in doc.items() if k != "identity_sha256"}):
        bad.append("identity digest does not match its contents")
    if doc.get("config_sha256") != _sha(doc.get("config")):
        bad.append("config digest does not match the config")
    if doc.get("package_sha256") != package_digest():
        bad.append("the installed package differs from the one the identity names")
    return bad


def read_runs(path: str) -> list[dict]:
    out = []
    with open(path) as f:
        for line in f:
            line = line.strip()
            if line.startswith("{"):
                d = json.loads(line)
                if "value" in d and "metric" in d and d.get("impl", "ours") != "reference":
                    out.append(d)
    return out


def summarize(on: list[dict], off: list[dict], bound_pct: Optional[float] = None,
              identity: Optional[dict] = None) -> dict:
    issues = []
    runs = on + off
    if not on or not off:
        issues.append("need at least one checked and one unchecked run")
    for key in ("metric", "n_gpus", "dtype"):
        vals = {json.dumps(r.get(key), sort_keys=True) for r in runs}
        if len(vals) > 1:
            issues.append(f"runs differ in {key}")
    cfgs = {_sha(r.get("config")) for r in runs}
    if len(cfgs) > 1:
        issues.append("runs differ in config")
    if identity is not None:
        issues += validate_identity(identity)
        if runs and identity.get("config") is not None and _sha(runs[0].get("config")) != identity["config_sha256"]:
            issues.append("runs were not made with the identity's config")
    res = {"schema": "sdcguard_b200.overhead.v1", "on_runs": len(on), "off_runs": len(off), "issues": issues,
           "measurement_sha256": _sha({"on": on, "off": off})}
    if on and off:
        hib = runs[0].get("higher_is_better", True)
        mon, moff = statistics.median(r["value"] for r in on), statistics.median(r["value"] for r in off)
        ovh = (1 - mon / moff) if hib else (mon / moff - 1)
        ratios = [(1 - a["value"] / b["value"]) if hib else (a["value"] / b["value"] - 1) for a in on for b in off]
        res.update(on_median=mon, off_median=moff, overhead_pct=round(100 * ovh, 2),
                   overhead_pct_range=[round(100 * min(ratios), 2), round(100 * max(ratios), 2)],
                   unit=runs[0].get("unit"))
    ident_ok = not issues
    fs = [catalog.finding("overhead.identity", "satisfied" if ident_ok else "unknown",
                          "runs are matched" if ident_ok else issues[0], "bench lines and identity document")]
    if bound_pct is not None and "overhead_pct" in res:
        ok = res["overhead_pct"] <= bound_pct and ident_ok
        fs.append(catalog.finding("overhead.bound", ("satisfied" if ok else "violated") if ident_ok else "unknown",
                                  f"overhead {res['overhead_pct']}% against a bound of {bound_pct}%",
                                  "median of matched runs", {"overhead_pct": res["overhead_pct"],
                                                             "bound_pct": bound_pct}))
    res["findings"] = fs
    res["verdict"] = "PASS" if all(f["verdict"] == "satisfied" for f in fs) else (
        "FAIL" if any(f["verdict"] == "violated" for f in fs) else "HOLD")
    return res


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="sdcguard overhead")
    sub = ap.add_subparsers(dest="cmd", required=True)
    p = sub.add_parser("prepare")
    p.add_argument("--config", required=True)
    p.add_argument("--model-dir")
    p.add_argument("--gpu-uuid", required=True)
    p.add_argument("--out", required=True)
    c = sub.add_parser("compare")
    c.add_argument("identity", nargs="?")
    c.add_argument("--on", required=True)
    c.add_argument("--off", required=True)
    c.add_argument("--bound", type=float)
    c.add_argument("--json", action="store_true")
    a = ap.parse_args(argv)
    if a.cmd == "prepare":
        with open(a.config) as f:
            cfg = json.load(f)
        try:
            doc = prepare_identity(cfg, a.model_dir, a.gpu_uuid)
        except (OSError, ValueError) as e:
            print(f"overhead: {e}", file=sys.stderr)
            return 2
        with open(a.out, "w") as f:
            json.dump(doc, f, indent=1, sort_keys=True)
        print(f"identity {doc['identity_sha256'][:16]} written to {a.out}")
        return 0
    ident = None
    if a.identity:
        with open(a.identity) as f:
            ident = json.load(f)
    r = summarize(read_runs(a.on), read_runs(a.off), a.bound, ident)
    if a.json:
        print(json.dumps(r, indent=1))
    else:
        if "overhead_pct" in r:
            print(f"overhead {r['overhead_pct']}% (range {r['overhead_pct_range']}) on {r['on_median']:.1f} vs "
                  f"{r['off_median']:.1f} {r['unit']}")
        for i in r["issues"]:
            print(f"  issue: {i}")
        print(r["verdict"])
    return {"PASS": 0, "HOLD": 1, "FAIL": 3}[r["verdict"]]


if __name__ == "__main__":
    raise SystemExit(main())
