"""Portable evidence bundle of an assessment: the recording, the lifetime events and the assessment, with a manifest
of SHA-256 digests, verifiable offline; optionally signed with a certify key.

    python -m sdcguard_b200.evidence.bundle create OUT --recording DIR --events ev.jsonl [--key fleet.key]
    python -m sdcguard_b200.evidence.bundle verify OUT [--pubkey fleet.pub]
    python -m sdcguard_b200.evidence.bundle report OUT          # OUT/report.html

create copies only the files it is given (regular files, at most 64 MiB each, 512 MiB in total), re-runs the
assessment on the copies, and writes manifest.json {format, files: {path: {sha256, bytes}}, assessment,
assessment_sha256}. verify recomputes every digest, checks no file was added or removed, re-runs the assessment on
the bundle's own copies and compares verdicts. Digests are local integrity; a signature (with a key) says who made
the bundle, not that the recording is true.

Reference: src/sdcguard/assessment_bundle.py:1-25 (copy rules, limits, offline verification; `create_bundle` :226,
`verify_bundle` :370).
"""
from __future__ import annotations

import argparse
import base64
import hashlib
import html
import json
import os
import shutil
from typing import Optional

from .assessment import assess

FORMAT = "sdcguard-b200-evidence-bundle/1"
MANIFEST = "manifest.json"
MAX_FILE = 64 << 20
MAX_TOTAL = 512 << 20


def _sha(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def _canon(d: dict) -> bytes:
    return json.dumps(d, sort_keys=True, separators=(",", ":"), default=str).encode()


def _files(root: str) -> list[str]:
    out = []
    for d, _, fs in os.walk(root):
        for f in fs:
            p = os.path.relpath(os.path.join(d, f), root)
            if p != MANIFEST:
                out.append(p)
    return sorted(out)


def create(out: str, recording: str, events: Optional[str] = None, key: Optional[str] = None) -> dict:
    if os.path.exists(out) and os.listdir(out):
        raise FileExistsError(f"{out} is not empty")
    os.makedirs(os.path.join(out, "recording"), exist_ok=True)
    total = 0
    for f in sorted(os.listdir(recording)):
        src = os.path.join(recording, f)
        if not os.path.isfile(src) or os.path.islink(src):
            continue
        n = os.path.getsize(src)
        total += n
        if n > MAX_FILE or total > MAX_TOTAL:
            raise ValueError(f"{src}: over the bundle's size limits")
        shutil.copyfile(src, os.path.join(out, "recording", f))
    ev = None
    if events:
        ev = os.path.join(out, "lifetime.jsonl")
        shutil.copyfile(events, ev)
    a = assess(os.path.join(out, "recording"), ev)
    a["recording"] = "recording"
    man = {"format": FORMAT, "files": {p: {"sha256": _sha(os.path.join(out, p)),
                                           "bytes": os.path.getsize(os.path.join(out, p))} for p in _files(out)},
           "assessment": a, "assessment_sha256": hashlib.sha256(_canon(a)).hexdigest(),
           "integrity": "local SHA-256 consistency" + (" and an Ed25519 signature" if key else "")}
    if key:
        from ..tools.certify import _crypto, key_id
        ser, _, _ = _crypto()
        with open(key, "rb") as f:
            k = ser.load_pem_private_key(f.read(), password=None)
        man["key_id"] = key_id(k.public_key())
        man["signature"] = base64.b64encode(k.sign(_canon({x: y for x, y in man.items() if x != "signature"}))).decode()
    with open(os.path.join(out, MANIFEST), "w") as f:
        json.dump(man, f, indent=1)
    return man


def verify(out: str, pubkey: Optional[str] = None) -> dict:
    with open(os.path.join(out, MANIFEST)) as f:
        man = json.load(f)
    problems = []
    if man.get("format") != FORMAT:
        problems.append("unknown format")
    listed, present = set(man.get("files", {})), set(_files(out))
    problems += [f"missing: {p}" for p in sorted(listed - present)]
    problems += [f"not in the manifest: {p}" for p in sorted(present - listed)]
    for p in sorted(listed & present):
        if _sha(os.path.join(out, p)) != man["files"][p]["sha256"]:
            problems.append(f"changed: {p}")
    if hashlib.sha256(_canon(man.get("assessment", {}))).hexdigest() != man.get("assessment_sha256"):
        problems.append("assessment changed")
    ev = os.path.join(out, "lifetime.jsonl")
    again = assess(os.path.join(out, "recording"), ev if os.path.exists(ev) else None)
    if again["verdict"] != man.get("assessment", {}).get("verdict"):
        problems.append(f"re-assessment gives {again['verdict']}, the manifest says "
                        f"{man.get('assessment', {}).get('verdict')}")
    if pubkey:
        from ..tools.certify import _crypto, key_id
        ser, _, _ = _crypto()
        with open(pubkey, "rb") as f:
            pub = ser.load_pem_public_key(f.read())
        if man.get("key_id") != key_id(pub):
            problems.append("signed with another key (or unsigned)")
        else:
            try:
                pub.verify(base64.b64decode(man["signature"]), _canon({x: y for x, y in man.items() if x != "signature"}))
            except Exception:  # noqa: BLE001
                problems.append("bad signature")
    return {"valid": not problems, "problems": problems, "verdict": man.get("assessment", {}).get("verdict")}


def report(out: str) -> str:
    with open(os.path.join(out, MANIFEST)) as f:
        man = json.load(f)
    a = man["assessment"]
    e = html.escape
    rows = "".join(f"<tr><td>{e(p)}</td><td>{v['bytes']}</td><td><code>{v['sha256'][:16]}</code></td></tr>"
                   for p, v in sorted(man["files"].items()))
    viol = "".join(f"<li>{e(v['rule'])} at event {v['step']}: {e(v['message'])}</li>" for v in a["lifetime"]["violations"])
    page = (f"<!doctype html><meta charset='utf-8'><title>Assessment</title><h1>{e(a['verdict'])}</h1>"
            f"<p>Scope: {e(a['scope'])}</p><h2>Coverage</h2><pre>{e(json.dumps(a['coverage'], indent=1))}</pre>"
            f"<h2>Lifetime</h2><p>{a['lifetime']['events']} events</p><ul>{viol or '<li>no rule broken</li>'}</ul>"
            f"<h2>Files</h2><table>{rows}</table><p>{e(man['integrity'])}</p>")
    p = os.path.join(out, "report.html")
    with open(p, "w") as f:
        f.write(page)
    return p


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m sdcguard_b200.evidence.bundle")
    sub = ap.add_subparsers(dest="cmd", required=True)
    c = sub.add_parser("create")
    c.add_argument("out")
    c.add_argument("--recording", required=True)
    c.add_argument("--events")
    c.add_argument("--key")
    v = sub.add_parser("verify")
    v.add_argument("out")
    v.add_argument("--pubkey")
    r = sub.add_parser("report")
    r.add_argument("out")
    a = ap.parse_args(argv)
    if a.cmd == "create":
        m = create(a.out, a.recording, a.events, a.key)
        print(json.dumps({"verdict": m["assessment"]["verdict"], "files": len(m["files"])}))
        return 0
    if a.cmd == "verify":
        res = verify(a.out, a.pubkey)
        print(json.dumps(res))
        return 0 if res["valid"] else 1
    print(report(a.out))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
