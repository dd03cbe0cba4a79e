"""Offline evidence packets of the KV-checksum coverage layer, and their command lines:

    sdcguard checksum-observer inspect SNAPSHOT.json [--json]
    sdcguard checksum-observer capture --snapshot SNAPSHOT.json --out PACKET
    sdcguard checksum-client   inspect --plan P --inventory I --captures C [--json]
    sdcguard checksum-client   capture --plan P --inventory I --captures C --out PACKET
    sdcguard native-checks     capture --owner-result DIR --out PACKET [--require checksum|lease ...]
    sdcguard {checksum-observer,checksum-client,native-checks} verify PACKET [--json]

`inspect` evaluates saved inputs and prints the report. `capture` writes a packet: the inputs byte for byte under
inputs/, the report as report.json and report.txt, and manifest.json naming the packet's schema and the SHA-256 of
every file. `verify` re-hashes every file against the manifest, recomputes the report from the retained inputs
and requires it to equal the retained report byte for byte. Inputs are read through the bounded, strict readers of
`coverage.evidence`; the evaluators are `observer.snapshot_report`, `client.evaluate` and the coverage gate
(`gate.inspect`), so the packets say what the gate says.

Release semantics: the observer and client reports never release anything (exit 2, HOLD: they describe coverage of
a recording, not a qualified runtime); native-checks exits 0 only when the owner result passes the required checks.
Local hashes establish the packet's consistency, not who recorded it.

Reference: src/sdcguard/checksum_observer_report.py (:318), checksum_client_report.py (:124), native_checks.py
(:634): the same commands and exit codes; the packet layout here is this package's own.
"""
from __future__ import annotations

import argparse
import json
import os
import shutil
import sys
from pathlib import Path

from . import evidence as ev

MANIFEST = "manifest.json"
PACKETS = {"checksum-observer": "sdcguard_b200.checksum-observer-packet.v1",
           "checksum-client": "sdcguard_b200.checksum-client-packet.v1",
           "native-checks": "sdcguard_b200.native-checks-packet.v1"}
CLIENT_INPUTS = ("REQUEST_PLAN.json", "CLIENT_INVENTORY.json", "CAPTURES.json")


def _read(path: str, limit: int = ev.MAX_FILE_BYTES) -> bytes:
    p = Path(path).absolute()
    return ev.read_file(p.parent, p.name, limit)


# ------------------------------------------------------------------------------------------ evaluators
def observer_report(raw: bytes) -> dict:
    from .observer import snapshot_report
    return {"kind": "checksum-observer", "release": "HOLD", **snapshot_report(ev.parse_json(raw))}


def client_report(plan: bytes, inventory: bytes, captures: bytes) -> dict:
    from .client import evaluate
    return {"kind": "checksum-client", "release": "HOLD", **evaluate(plan, inventory, captures)}


def native_report(owner_dir: str, required: list) -> dict:
    """Engine pass vs actually covered: the gate's per-request rows over the owner result, with the requests whose
    engine reported a pass while the required coverage is incomplete listed apart."""
    from .gate import inspect
    ans = inspect(owner_dir, required)
    rows = ans.get("requests") or []
    not_covered = [r for r in rows if r.get("decision") == "HOLD" and
                   any(((r.get("checks") or {}).get(c) or {}).get("native_result") == "passed" for c in required)]
    return {"kind": "native-checks", "release": ans.get("decision"), "required": required,
            "engine_pass_not_covered": len(not_covered), "gate": ans}


def render(rep: dict) -> str:
    lines = [f"{rep['kind']}: release {rep.get('release')}"]
    summ = rep.get("summary") or (rep.get("gate") or {}).get("summary")
    if isinstance(summ, dict):
        lines.append("Summary:")
        lines += [f"  {k}: {json.dumps(v, sort_keys=True)}" for k, v in summ.items()]
    if rep["kind"] == "native-checks":
        lines.append(f"Engine pass, not covered: {rep['engine_pass_not_covered']} request(s)")
    holds = rep.get("hold_reasons") or (rep.get("gate") or {}).get("hold_reasons") or []
    if holds:
        lines.append("Hold reasons:")
        lines += [f"* {h}" for h in holds]
    lines.append("Local hashes establish consistency, not who recorded the evidence.")
    return "\n".join(lines) + "\n"


# ------------------------------------------------------------------------------------------ packets
def _write_packet(out: str, kind: str, inputs: dict, rep: dict) -> dict:
    outp = Path(out).absolute()
    if outp.exists():
        raise ev.EvidenceError(f"{out} exists: a packet is written once")
    tmp = outp.with_name(outp.name + ".partial")
    if tmp.exists():
        shutil.rmtree(tmp)
    (tmp / "inputs").mkdir(parents=True)
    files = {f"inputs/{n}": raw for n, raw in inputs.items()}
    files["report.json"] = ev.json_bytes(rep)
    files["report.txt"] = render(rep).encode()
    for name, raw in files.items():
        (tmp / name).parent.mkdir(parents=True, exist_ok=True)
        (tmp / name).write_bytes(raw)
    manifest = {"schema": PACKETS[kind], "files": {n: ev.digest(raw) for n, raw in sorted(files.items())}}
    (tmp / MANIFEST).write_bytes(ev.json_bytes(manifest))
    os.replace(tmp, outp)
    return rep


def _load_packet(path: str, kind: str) -> dict:
    root = Path(path).absolute()
    manifest = ev.parse_json(ev.read_file(root, MANIFEST))
    if type(manifest) is not dict or manifest.get("schema") != PACKETS[kind]:
        raise ev.EvidenceError(f"not a {kind} packet")
    names = manifest.get("files")
    if type(names) is not dict or not names:
        raise ev.EvidenceError("packet manifest lists no files")
    files = {}
    for name, want in names.items():
        raw = ev.read_file(root, name)
        if ev.digest(raw) != want:
            raise ev.EvidenceError(f"{name} does not match its manifest hash")
        files[name] = raw
    on_disk = {str(p.relative_to(root)) for p in root.rglob("*") if p.is_file()} - {MANIFEST}
    if on_disk != set(names):
        raise ev.EvidenceError("packet holds files its manifest does not list, or lacks listed ones")
    return files


def verify(path: str, kind: str) -> dict:
    files = _load_packet(path, kind)
    if kind == "checksum-observer":
        rep = observer_report(files["inputs/SNAPSHOT.json"])
    elif kind == "checksum-client":
        rep = client_report(*(files[f"inputs/{n}"] for n in CLIENT_INPUTS))
    else:
        import tempfile
        retained = json.loads(files["report.json"])
        with tempfile.TemporaryDirectory(prefix="sdcguard_native_") as tmp:
            for name, raw in files.items():
                if name.startswith("inputs/owner/"):
                    p = Path(tmp) / name[len("inputs/owner/"):]
                    p.parent.mkdir(parents=True, exist_ok=True)
                    p.write_bytes(raw)
            rep = native_report(tmp, retained.get("required") or [])
    if ev.json_bytes(rep) != files["report.json"] or render(rep).encode() != files["report.txt"]:
        raise ev.EvidenceError("the retained report differs from the one recomputed from the retained inputs")
    return rep


def _owner_files(owner_dir: str) -> dict:
    root = Path(owner_dir).absolute()
    out = {}
    for p in sorted(root.rglob("*")):
        if p.is_file():
            rel = str(p.relative_to(root))
            out[f"owner/{rel}"] = ev.read_file(root, rel)
    if not out:
        raise ev.EvidenceError(f"{owner_dir}: no owner-result files")
    return out


# ------------------------------------------------------------------------------------------ command lines
def _cli(kind: str, argv) -> int:
    ap = argparse.ArgumentParser(prog=f"sdcguard {kind}")
    sub = ap.add_subparsers(dest="cmd", required=True)
    if kind == "checksum-observer":
        p = sub.add_parser("inspect")
        p.add_argument("snapshot")
        p = sub.add_parser("capture")
        p.add_argument("--snapshot", required=True)
        p.add_argument("--out", required=True)
    elif kind == "checksum-client":
        for name in ("inspect", "capture"):
            p = sub.add_parser(name)
            p.add_argument("--plan", required=True)
            p.add_argument("--inventory", required=True)
            p.add_argument("--captures", required=True)
            if name == "capture":
                p.add_argument("--out", required=True)
    else:
        p = sub.add_parser("capture")
        p.add_argument("--owner-result", required=True)
        p.add_argument("--out", required=True)
        p.add_argument("--require", choices=("lease", "checksum"), action="append", default=None)
    v = sub.add_parser("verify")
    v.add_argument("packet")
    for s in sub.choices.values():
        s.add_argument("--json", action="store_true")
    a = ap.parse_args(argv)
    try:
        if a.cmd == "verify":
            rep = verify(a.packet, kind)
        elif kind == "checksum-observer":
            raw = _read(a.snapshot)
            rep = observer_report(raw)
            if a.cmd == "capture":
                _write_packet(a.out, kind, {"SNAPSHOT.json": raw}, rep)
        elif kind == "checksum-client":
            raws = tuple(_read(x) for x in (a.plan, a.inventory, a.captures))
            rep = client_report(*raws)
            if a.cmd == "capture":
                _write_packet(a.out, kind, dict(zip(CLIENT_INPUTS, raws)), rep)
        else:
            required = list(dict.fromkeys(a.require or ["checksum"]))
            rep = native_report(a.owner_result, required)
            _write_packet(a.out, kind, _owner_files(a.owner_result), rep)
    except (ValueError, OSError, KeyError, TypeError) as e:
        print(f"{kind}: evidence is inconclusive: {e}")
        return 2
    sys.stdout.write(ev.json_bytes(rep).decode() + "\n" if a.json else render(rep))
    if kind == "native-checks":
        return 0 if rep.get("release") == "PASS" else 2
    return 2


def observer_main(argv=None) -> int:
    return _cli("checksum-observer", list(sys.argv[1:] if argv is None else argv))


def client_main(argv=None) -> int:
    return _cli("checksum-client", list(sys.argv[1:] if argv is None else argv))


def native_main(argv=None) -> int:
    return _cli("native-checks", list(sys.argv[1:] if argv is None else argv))
