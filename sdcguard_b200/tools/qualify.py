"""Qualify a serving-stack change: start a baseline and a candidate server, run the same probes against both, and
write the evidence `decide` needs.

    python -m sdcguard_b200.tools.qualify --out qual/ \\
        --baseline "python -m sdcguard_b200.serve.http --model tiny --port 8101" --baseline-url http://127.0.0.1:8101 \\
        --candidate "python -m sdcguard_b200.serve.http --model tiny --precision fp8 --port 8102" \\
        --candidate-url http://127.0.0.1:8102

Per server: ready (with a probe), perf, isolation and consistency, plus its metrics at the end (what it checked) and
its stack record. Servers start one after the other on the same GPU (each is stopped, by its own PID, before the next
starts), so they never compete for it. Then `decide` runs on the collected files and its decision is written next
to them.

Reference: src/sdcguard/qualify.py (`Server` :87, `run_one` :157).
"""
from __future__ import annotations

import argparse
import json
import os
import shlex
import signal
import subprocess
import time
from typing import Optional

from . import _client, consistency, isolation, perf, ready


class Server:
    """A server subprocess in its own process group; stop() ends exactly that group."""

    def __init__(self, cmd: str, url: str, log: str, start_timeout: float = 600.0):
        self.url = url
        self.logf = open(log, "w")
        self.p = subprocess.Popen(shlex.split(cmd), stdout=self.logf, stderr=subprocess.STDOUT,
                                  start_new_session=True)
        t_end = time.time() + start_timeout
        while time.time() < t_end:
            if self.p.poll() is not None:
                raise RuntimeError(f"server exited with {self.p.returncode} (log: {log})")
            try:
                if json.loads(_client.get(url.rstrip("/") + "/health", 2.0)).get("ok"):
                    return
            except Exception:  # noqa: BLE001  (not up yet)
                pass
            time.sleep(1.0)
        self.stop()
        raise RuntimeError(f"server did not come up in {start_timeout:.0f} s (log: {log})")

    def stop(self) -> None:
        if self.p.poll() is None:
            os.killpg(self.p.pid, signal.SIGTERM)
            try:
                self.p.wait(timeout=60)
            except subprocess.TimeoutExpired:
                os.killpg(self.p.pid, signal.SIGKILL)
                self.p.wait(timeout=30)
        self.logf.close()


def run_one(name: str, cmd: str, url: str, out: str, seconds: float = 10.0, clients: int = 8) -> dict:
    srv = Server(cmd, url, os.path.join(out, f"{name}.log"))
    try:
        res = {"ready": ready.check(url, probe=True), "perf": perf.run(url, clients=clients, seconds=seconds),
               "isolation": isolation.run(url), "consistency": consistency.run(url)}
        res["metrics"] = _client.get(url.rstrip("/") + "/metrics")
        res["stack"] = ready._stack(_client.parse_metrics(res["metrics"]))
    finally:
        srv.stop()
    with open(os.path.join(out, f"{name}.json"), "w") as f:
        json.dump(res, f, indent=1)
    return res


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m sdcguard_b200.tools.qualify")
    ap.add_argument("--out", required=True)
    ap.add_argument("--baseline", required=True)
    ap.add_argument("--baseline-url", required=True)
    ap.add_argument("--candidate", required=True)
    ap.add_argument("--candidate-url", required=True)
    ap.add_argument("--seconds", type=float, default=10.0)
    ap.add_argument("--policy")
    a = ap.parse_args(argv)
    os.makedirs(a.out, exist_ok=True)
    base = run_one("baseline", a.baseline, a.baseline_url, a.out, a.seconds)
    cand = run_one("candidate", a.candidate, a.candidate_url, a.out, a.seconds)
    from . import decide
    policy: Optional[dict] = None
    if a.policy:
        with open(a.policy) as f:
            policy = json.load(f)
    d = decide.decide(base, cand, policy)
    with open(os.path.join(a.out, "decision.json"), "w") as f:
        json.dump(d, f, indent=1)
    print(json.dumps({"decision": d["decision"], "sections": {k: v["verdict"] for k, v in d["sections"].items()}}))
    return 0 if d["decision"] == "ACCEPT" else 1


if __name__ == "__main__":
    raise SystemExit(main())
