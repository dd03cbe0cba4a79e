"""Bind a local model directory to stable digests before the engine starts, and check it again later.

    python -m sdcguard_b200.evidence.model_reference capture MODEL_DIR --out REF.json
    python -m sdcguard_b200.evidence.model_reference observe REF.json MODEL_DIR
    sdcguard model-ref ...

capture hashes every regular file under the directory (relative path, size, SHA-256; symbolic links and special
files are refused, at most 4096 files and 2 TB) and digests the sorted listing (`capture_sha256`). bind adds the
model id the operator names. observe re-hashes the directory and reports every added, removed or changed file. A
matching observation is local consistency of the files, not proof of the weights the engine loaded.

Reference: src/sdcguard/model_reference.py:1-10 (`capture`, `bind`, `observe`, `validate_capsule`).
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import stat
import sys

from . import catalog

SCHEMA = "sdcguard_b200.model-reference.v1"
MAX_FILES = 4096
MAX_TOTAL = 2 << 40


class ModelReferenceError(ValueError):
    pass


def _hash_file(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(16 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def capture(model_dir: str) -> dict:
    root = os.path.abspath(model_dir)
    files, total = [], 0
    for d, dirs, names in os.walk(root, followlinks=False):
        dirs.sort()
        for n in sorted(names):
            p = os.path.join(d, n)
            st = os.lstat(p)
            if not stat.S_ISREG(st.st_mode):
                raise ModelReferenceError(f"{os.path.relpath(p, root)}: not a regular file")
            total += st.st_size
            if len(files) >= MAX_FILES or total > MAX_TOTAL:
                raise ModelReferenceError("model directory exceeds the capture limits")
            files.append({"path": os.path.relpath(p, root), "bytes": st.st_size, "sha256": _hash_file(p)})
    files.sort(key=lambda f: f["path"])
    if not files:
        raise ModelReferenceError("model directory holds no files")
    listing = json.dumps(files, sort_keys=True, separators=(",", ":")).encode()
    return {"schema": SCHEMA, "files": files, "total_bytes": total, "capture_sha256": hashlib.sha256(listing).hexdigest()}


def validate_capsule(ref: dict) -> None:
    if not isinstance(ref, dict) or ref.get("schema") != SCHEMA or not isinstance(ref.get("files"), list):
        raise ModelReferenceError(f"not a {SCHEMA} document")
    listing = json.dumps(ref["files"], sort_keys=True, separators=(",", ":")).encode()
    if hashlib.sha256(listing).hexdigest() != ref.get("capture_sha256"):
        raise ModelReferenceError("capture digest does not match the file listing")


def bind(ref: dict, model_id: str) -> dict:
    validate_capsule(ref)
    return {**ref, "model_id": model_id}


def observe(ref: dict, model_dir: str) -> dict:
    validate_capsule(ref)
    try:
        now = capture(model_dir)
    except (OSError, ModelReferenceError) as e:
        f = catalog.finding("model.reference", "unknown", f"directory not captured: {e}", "local files")
        return {"match": False, "added": [], "removed": [], "changed": [], "findings": [f], "verdict": "HOLD"}
    old = {f["path"]: f for f in ref["files"]}
    new = {f["path"]: f for f in now["files"]}
    added = sorted(set(new) - set(old))
    removed = sorted(set(old) - set(new))
    changed = sorted(p for p in set(old) & set(new) if old[p]["sha256"] != new[p]["sha256"])
    match = not (added or removed or changed)
    f = catalog.finding("model.reference", "satisfied" if match else "violated",
                        "the files hash to the bound reference" if match else
                        f"{len(added)} added, {len(removed)} removed, {len(changed)} changed file(s)", "local files",
                        {"capture_sha256": now["capture_sha256"], "model_id": ref.get("model_id")})
    return {"match": match, "added": added, "removed": removed, "changed": changed, "findings": [f],
            "verdict": "PASS" if match else "FAIL"}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="sdcguard model-ref")
    sub = ap.add_subparsers(dest="cmd", required=True)
    c = sub.add_parser("capture")
    c.add_argument("model_dir")
    c.add_argument("--out", required=True)
    c.add_argument("--model-id")
    o = sub.add_parser("observe")
    o.add_argument("ref")
    o.add_argument("model_dir")
    o.add_argument("--json", action="store_true")
    a = ap.parse_args(argv)
    try:
        if a.cmd == "capture":
            ref = capture(a.model_dir)
            if a.model_id:
                ref = bind(ref, a.model_id)
            with open(a.out, "w") as f:
                json.dump(ref, f, indent=1, sort_keys=True)
            print(f"captured {len(ref['files'])} files, {ref['capture_sha256'][:16]}")
            return 0
        with open(a.ref) as f:
            ref = json.load(f)
        r = observe(ref, a.model_dir)
    except (OSError, ModelReferenceError) as e:
        print(f"model-ref: {e}", file=sys.stderr)
        return 2
    print(json.dumps(r, indent=1) if a.json else f"{r['verdict']}: {r['findings'][0]['message']}")
    return 0 if r["match"] else 1


if __name__ == "__main__":
    raise SystemExit(main())
