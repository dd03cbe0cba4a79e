"""`sdcguard nhc`: node health check built on `sdcguard check`, for schedulers and node-problem detectors.

    sdcguard nhc [--seconds 60] [--out nhc_out] [--devices 0,1,...]     # run the check on every GPU
    sdcguard nhc --cached [--max-age-hours 24]                           # report the last result instantly

One line on stdout; exit 0 = OK, 1 = a GPU computed wrong results, 2 = could not tell (the conventions of
node-problem-detector custom plugins). Each GPU's check runs in its own process group with a deadline of
1.5 x its budget + 600 s; at the deadline, or on an interrupt, the whole group is killed, so a hung GPU cannot hold
the node. The result goes to OUT/status.json. A FAIL sticks: a later check that cannot finish reports the FAIL
again, and only a clean check clears it. `--cached` never runs anything (for health-check hooks with a short time
limit, such as Slurm's HealthCheckProgram); it reports the cached FAIL at any age, and an OK older than
--max-age-hours as UNKNOWN. `--simulate-faults` prints what a FAIL line looks like, runs nothing and never touches
the cached status. The GPUs' checks run at the same time.

Reference: src/sdcguard/cli.py:65-106 (deadline and process-group kill around a check), :228-330 (`cmd_nhc`: one
line, exit codes, sticky FAIL, the cached mode and its status.json record, whose three fields are kept).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import signal
import subprocess
import sys
import tempfile
import threading
import time
from dataclasses import dataclass
from typing import Callable, Optional


def deadline(seconds: float) -> float:
    """How long a check may run before it counts as hung: its budget, room for loading and the slowest phase."""
    return float(seconds) * 1.5 + 600.0


def _stop_group(p: subprocess.Popen) -> None:
    try:
        os.killpg(p.pid, signal.SIGKILL)
    except (ProcessLookupError, PermissionError):
        pass


def check_command(device: str, seconds: float) -> list[str]:
    return [sys.executable, "-m", "sdcguard_b200.tools.check", "--device", device, "--seconds", str(seconds), "--json"]


def _finish(p: subprocess.Popen, t_end: float) -> dict:
    """Collect one check started by run_all: {"code", "result" (its JSON line, or None), "timed_out"}."""
    try:
        out, _ = p.communicate(timeout=max(0.0, t_end - time.monotonic()))
    except subprocess.TimeoutExpired:   # a hung GPU: nothing of the check outlives the deadline
        _stop_group(p)
        try:
            p.communicate(timeout=30)   # bounded: a process stuck in a driver call dies when the call returns
        except subprocess.TimeoutExpired:
            pass
        return {"code": None, "result": None, "timed_out": True}
    _stop_group(p)                      # a worker left behind by a check that crashed
    res = None
    for line in reversed((out or "").splitlines()):
        line = line.strip()
        if line.startswith("{"):
            try:
                res = json.loads(line)
                break
            except ValueError:
                pass
    return {"code": p.returncode, "result": res, "timed_out": False}


def run_all(cmds: list[list[str]], limit: float) -> list[dict]:
    """Every GPU's check at once, each in its own process group, all under one deadline. Each check's output is
    drained by a thread of its own, so a check that writes a lot of log never blocks on a full pipe while another
    one is being waited for (a healthy check must not look hung)."""
    t_end = time.monotonic() + limit
    procs = [subprocess.Popen(c, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True, start_new_session=True)
             for c in cmds]
    results: list[Optional[dict]] = [None] * len(procs)

    def collect(i: int) -> None:
        results[i] = _finish(procs[i], t_end)

    workers = [threading.Thread(target=collect, args=(i,), daemon=True) for i in range(len(procs))]
    try:
        for w in workers:
            w.start()
        for w in workers:
            while w.is_alive():
                w.join(timeout=0.5)
    except BaseException:               # an interrupt: stop every group, then let it propagate
        for p in procs:
            _stop_group(p)
        raise
    return [r if r is not None else {"code": None, "result": None, "timed_out": True} for r in results]


@dataclass
class NodeStatus:
    """The node's last health line, kept in OUT/status.json as {"time", "code", "line"} (the file the scheduler's
    cached health hook reads). A FAIL (code 1) outlives any number of checks that could not finish; only a clean
    check replaces it."""

    line: str
    code: int
    time: float

    NAME = "status.json"

    @classmethod
    def load(cls, out: str) -> Optional["NodeStatus"]:
        try:
            with open(os.path.join(out, cls.NAME)) as f:
                raw = json.load(f)
        except (OSError, ValueError):
            return None
        if not isinstance(raw, dict):
            return None
        return cls(line=str(raw.get("line", "")), code=raw.get("code"), time=raw.get("time"))

    def store(self, out: str) -> None:
        """Replace the file atomically (a reader never sees half a record); a read-only OUT is not an error."""
        try:
            os.makedirs(out, exist_ok=True)
            fd, tmp = tempfile.mkstemp(dir=out, prefix=".status.")
            with os.fdopen(fd, "w") as f:
                json.dump({"time": self.time, "code": self.code, "line": self.line}, f)
            os.replace(tmp, os.path.join(out, self.NAME))
        except OSError:
            pass

    def age_hours(self, now: float) -> Optional[float]:
        try:
            h = (now - float(self.time)) / 3600.0
        except (TypeError, ValueError):
            return None
        return h if math.isfinite(h) and h >= 0 else None

    def carry_fail(self, line: str, code: int) -> tuple[str, int]:
        """What to report when a new check ended with (line, code): an inconclusive result keeps a recorded FAIL."""
        if code == 2 and self.code == 1:
            return f"{self.line or 'FAIL'} (a later check: {line})", 1
        return line, code

    def cached_report(self, max_age_hours: float, now: float, out: str) -> tuple[str, int]:
        age = self.age_hours(now)
        if age is None:
            return f"UNKNOWN: unreadable sdcguard check result in {out}", 2
        if self.code == 1:
            return self.line or "FAIL", 1
        if age > max_age_hours:
            return f"UNKNOWN: last sdcguard check was {age:.0f} hours ago (limit {max_age_hours:g})", 2
        return self.line or "OK", self.code if self.code in (0, 2) else 2


def write_status(out: str, line: str, code: int) -> None:
    NodeStatus(line=line, code=code, time=time.time()).store(out)


def cached(out: str, max_age_hours: float) -> tuple[str, int]:
    """The cached mode: report the stored status, never run anything."""
    st = NodeStatus.load(out)
    if st is None:
        return f"UNKNOWN: no readable sdcguard check result in {out} yet", 2
    return st.cached_report(max_age_hours, time.time(), out)


def judge(devices: list[str], runs: list[dict], limit: float) -> tuple[str, int]:
    bad = [(d, r) for d, r in zip(devices, runs) if r["code"] == 1 or (r["result"] or {}).get("gemm_wrong", 0)
           or (r["result"] or {}).get("copies_wrong", 0)]
    if bad:
        d, r = bad[0]
        res = r["result"] or {}
        return (f"FAIL: {len(bad)} of {len(devices)} GPUs computed wrong results; first {d} "
                f"({res.get('gemm_wrong', '?')} GEMM, {res.get('copies_wrong', '?')} copy); worst z "
                f"{res.get('worst_z', '?')}"), 1
    hung = [d for d, r in zip(devices, runs) if r["timed_out"]]
    if hung:
        return f"UNKNOWN: the check on {', '.join(hung)} did not finish within {limit:.0f} s", 2
    odd = [d for d, r in zip(devices, runs) if r["code"] != 0 or r["result"] is None]
    if odd:
        return f"UNKNOWN: the check on {', '.join(odd)} exited without a result", 2
    checks = sum(int(r["result"].get("gemm_checks", 0)) for r in runs)
    worst = max(float(r["result"].get("worst_z", 0.0)) for r in runs)
    return f"OK: {len(devices)} GPUs, {checks} checked GEMMs, worst clean z {worst:.3f}", 0


def run_nhc(devices: list[str], seconds: float, out: str,
            command: Callable[[str, float], list[str]] = check_command, limit: Optional[float] = None) -> tuple[str, int]:
    limit = deadline(seconds) if limit is None else limit
    runs = run_all([command(d, seconds) for d in devices], limit)
    line, code = judge(devices, runs, limit)
    prev = NodeStatus.load(out)
    if prev is not None:
        line, code = prev.carry_fail(line, code)
    write_status(out, line, code)
    return line, code


def _devices(spec: Optional[str]) -> list[str]:
    if spec:
        return [f"cuda:{int(x)}" for x in spec.split(",") if x.strip()]
    try:
        import torch
        n = torch.cuda.device_count()
    except Exception:  # noqa: BLE001
        n = 0
    return [f"cuda:{i}" for i in range(n)]


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="sdcguard nhc")
    ap.add_argument("--seconds", type=float, default=60.0)
    ap.add_argument("--out", default="nhc_out")
    ap.add_argument("--devices", help="comma-separated GPU indices (default: every visible GPU)")
    ap.add_argument("--cached", action="store_true")
    ap.add_argument("--max-age-hours", type=float, default=24.0)
    ap.add_argument("--simulate-faults", action="store_true",
                    help="demonstration: report what a wrong result looks like; the cached status is not touched")
    a = ap.parse_args(argv)
    if a.cached:
        line, code = cached(a.out, a.max_age_hours)
        print(line)
        return code
    if a.simulate_faults:
        print("SIMULATED: FAIL: 1 of 1 GPUs computed wrong results (demonstration; cached status unchanged)")
        return 2
    devs = _devices(a.devices)
    if not devs:
        line, code = "UNKNOWN: no CUDA device visible", 2
        print(line)
        return code
    line, code = run_nhc(devs, a.seconds, a.out)
    print(line)
    return code


if __name__ == "__main__":
    raise SystemExit(main())
