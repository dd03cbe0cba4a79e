"""Supervised capture of this engine's KV-checksum coverage, then the gate: `sdcguard operator run`.

    sdcguard operator run --out DIR --require checksum [--preflight-only] [--deadline 900]

1. CPU preflight (no GPU work): the output is a new directory under an existing parent; the installed package's
   native library and its source files hash to a recorded build witness; the Python, torch and CUDA versions; the
   GPUs the recorder would use are visible. Written to DIR/CPU_PREFLIGHT.json; anything but PASS stops here.
2. The recorder (`sdcguard pd-record`: prefill and decode of grouped shared-prefix requests through this engine's
   P/D path, every KV page transfer checksummed, cached-prefix pages re-verified) runs as a child process in its own
   process group, with its output to DIR/recording and its log to DIR/RECORDER.log, under a deadline. The
   supervisor records its start and end, exit status, whether the deadline ended it (the whole process group is
   then killed) and that no process of the group is left: DIR/SUPERVISOR.json (the cleanup evidence).
3. The coverage gate over the recording (`coverage.own`), to DIR/GATE.json, printed; exit 0 on PASS, else 2.

Any failure is recorded as DIR/OPERATOR_ERROR.json with decision HOLD (exit 2): an incomplete capture never passes.

Reference: src/sdcguard/native_operator/command.py (`sdcguard operator run`), supervisor.py:26 and runtime.py:211
(the supervised two-process vLLM recorder). Here the recorder is this engine's own P/D path.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import platform
import signal
import subprocess
import sys
import time
from pathlib import Path


def _write(path: Path, obj) -> None:
    tmp = path.with_name(path.name + ".tmp")
    tmp.write_text(json.dumps(obj, indent=1, sort_keys=True, default=str))
    os.replace(tmp, path)


def build_witness() -> dict:
    """SHA-256 of the loaded native library and of every kernel source file of the installed package."""
    from .. import _native
    pkg = Path(_native.__file__).parent
    src = {p.name: hashlib.sha256(p.read_bytes()).hexdigest() for p in sorted((pkg / "csrc").glob("*"))
           if p.is_file()}
    lib = _native.LIB_PATH
    return {"library": hashlib.sha256(lib.read_bytes()).hexdigest() if lib.exists() else None,
            "sources": src, "sources_digest": hashlib.sha256(json.dumps(src, sort_keys=True).encode()).hexdigest()}


def preflight(out: Path, gpus: int = 1) -> dict:
    checks = {}
    checks["output_is_new"] = not out.exists() and not out.is_symlink() and out.parent.is_dir()
    try:
        w = build_witness()
        checks["native_library_built"] = w["library"] is not None
    except OSError as e:
        w = {"error": str(e)}
        checks["native_library_built"] = False
    try:
        import torch
        versions = {"python": platform.python_version(), "torch": torch.__version__, "cuda": torch.version.cuda}
        visible = torch.cuda.device_count() if torch.cuda.is_available() else 0
    except Exception as e:  # noqa: BLE001  (a failed import is a failed preflight)
        versions, visible = {"error": str(e)}, 0
    checks["gpus_visible"] = visible >= gpus
    failed = [k for k, ok in checks.items() if not ok]
    return {"schema": "sdcguard_b200.operator-preflight.v1", "status": "PASS" if not failed else "FAIL",
            "failure": failed or None, "checks": checks, "build": w, "versions": versions, "gpus_visible": visible,
            "gpus_needed": gpus, "time": time.time()}


def supervise(cmd: list, log: Path, deadline: float) -> dict:
    """Run cmd in its own process group; kill the group at the deadline; report exit, timing and leftovers."""
    t0 = time.time()
    with open(log, "wb") as f:
        p = subprocess.Popen(cmd, stdout=f, stderr=subprocess.STDOUT, start_new_session=True)
        timed_out = False
        try:
            rc = p.wait(timeout=deadline)
        except subprocess.TimeoutExpired:
            timed_out = True
            os.killpg(p.pid, signal.SIGKILL)
            rc = p.wait(timeout=60)
    left = _group_alive(p.pid)
    if left:
        try:
            os.killpg(p.pid, signal.SIGKILL)
        except ProcessLookupError:
            pass
    return {"command": cmd, "pid": p.pid, "start": t0, "end": time.time(), "seconds": round(time.time() - t0, 2),
            "exit_code": rc, "timed_out": timed_out, "group_left_running": left,
            "clean": (rc == 0 and not timed_out and not left)}


def _group_alive(pgid: int, wait: float = 5.0) -> bool:
    """Is any live (not zombie) process of the group left? Waits up to `wait` seconds for killed ones to go."""
    t0 = time.time()
    while True:
        alive = False
        try:
            for d in os.listdir("/proc"):
                if not d.isdigit():
                    continue
                try:
                    with open(f"/proc/{d}/stat") as f:
                        fields = f.read().rsplit(")", 1)[1].split()
                except OSError:
                    continue
                if int(fields[2]) == pgid and fields[0] != "Z":      # fields: state, ppid, pgrp, ...
                    alive = True
                    break
        except OSError:                                               # no /proc: ask the kernel about the group
            try:
                os.killpg(pgid, 0)
                alive = True
            except (ProcessLookupError, PermissionError):
                alive = False
        if not alive or time.time() - t0 > wait:
            return alive
        time.sleep(0.1)


def run(args) -> int:
    out = Path(args.out).expanduser().absolute()
    required = list(dict.fromkeys(args.require))
    if required != ["checksum"]:
        print("HOLD: this engine's recorder records KV checksums only; lease coverage is not recorded.")
        return 2
    pre = preflight(out)
    if not pre["checks"]["output_is_new"]:
        print("HOLD: output must be a new directory with an existing parent.")
        return 2
    out.mkdir(mode=0o700)
    _write(out / "CPU_PREFLIGHT.json", pre)
    if pre["status"] != "PASS":
        print(f"HOLD: CPU preflight did not pass: {pre['failure']}")
        return 2
    if args.preflight_only:
        print("CPU preflight passed. No recorder or GPU work was started.")
        return 0
    try:
        cmd = [sys.executable, "-m", "sdcguard_b200.cli", "pd-record", str(out / "recording"),
               "--groups", str(args.groups), "--per-group", str(args.per_group), "--verify-cached-prefix"]
        sup = supervise(cmd, out / "RECORDER.log", args.deadline)
        _write(out / "SUPERVISOR.json", sup)
        if not sup["clean"]:
            raise RuntimeError(f"recorder did not finish cleanly (exit {sup['exit_code']}, timed out "
                               f"{sup['timed_out']}, processes left {sup['group_left_running']})")
        from ..coverage.own import inspect
        ans = inspect(out / "recording")
        _write(out / "GATE.json", ans)
        print(json.dumps({"decision": ans.get("decision"), "hold_reasons": ans.get("hold_reasons")}))
        return 0 if ans.get("decision") == "PASS" else 2
    except (Exception, KeyboardInterrupt) as e:  # noqa: BLE001  (an incomplete capture is a HOLD, recorded)
        _write(out / "OPERATOR_ERROR.json", {"kind": type(e).__name__, "detail": str(e)[:1024], "decision": "HOLD"})
        print(f"HOLD: operator run is incomplete: {str(e)[:1024]}")
        return 2


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="sdcguard operator", description=__doc__.split("\n\n")[0])
    sub = ap.add_subparsers(dest="cmd", required=True)
    r = sub.add_parser("run")
    r.add_argument("--out", required=True)
    r.add_argument("--require", action="append", choices=("checksum", "lease"), required=True)
    r.add_argument("--preflight-only", action="store_true")
    r.add_argument("--deadline", type=float, default=900.0)
    r.add_argument("--groups", type=int, default=8)
    r.add_argument("--per-group", type=int, default=20)
    p = sub.add_parser("preflight")
    p.add_argument("--out", required=True)
    a = ap.parse_args(argv)
    if a.cmd == "preflight":
        rep = preflight(Path(a.out).expanduser().absolute())
        print(json.dumps(rep, default=str))
        return 0 if rep["status"] == "PASS" else 2
    return run(a)


if __name__ == "__main__":
    raise SystemExit(main())
