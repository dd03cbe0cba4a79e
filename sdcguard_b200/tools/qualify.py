"""Qualify serving-stack changes: serve the trusted stack and each candidate in turn, run the same probes against
each, and decide every candidate against the baseline.

    sdcguard qualify --out qual/ --baseline "--model tiny" \\
        --candidate fp8="--model tiny --precision fp8" [--candidate NAME="ARGS" ...] [--policy policy.json]

Each stack is the arguments after --serve-cmd (default: this package's server, `python -m sdcguard_b200.serve.http`);
qualify adds the port and the alert log. Servers run one after the other on the same GPU, each in its own process
group, stopped before the next starts. Per server, in its directory under DIR/runs/: `ready --probe`, the quality
probe (greedy completions of a fixed prompt set and their top-20 log-probabilities, teacher-forced), `perf`,
`isolation`, `consistency`, its alert log and its /metrics at the end (what it checked) and its server log.

The baseline's quality probe is the reference; with --repeat-baseline (the default when there are candidates) the
baseline is served a second time and scored against it, which measures the noise floor the candidates' quality
verdicts are judged against. Each candidate then gets `decide` with its own evidence and the baseline's perf and
consistency runs: DIR/decision_NAME.json and .txt. DIR/report.txt lists every candidate's decision and sections;
DIR/repro_NAME.sh reruns one candidate's qualification alone; DIR/tested_conditions.json records what was exercised
(model, longest prompt, tokens, concurrency; `ready --qualified` reads it from the decision). Results of an earlier
qualification in DIR are moved to DIR/earlier-TIME first.

Exit 0 when every candidate is ACCEPT, 1 when one is REJECT, 2 otherwise.

Reference: src/sdcguard/qualify.py:1-60 (the procedure and its outputs), `Server` :87, `run_one` :157, `write_repro`
:253, `tested_conditions` :359, `set_aside_earlier` :402.
"""
from __future__ import annotations

import argparse
import json
import os
import shlex
import signal
import socket
import subprocess
import sys
import time
from typing import Optional

from . import _client, consistency, decide, gate_model, isolation, perf, ready

SERVE_CMD = f"{sys.executable} -m sdcguard_b200.serve.http"


def free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class Server:
    """A server subprocess in its own process group; stop() ends exactly that group."""

    def __init__(self, cmd: str, url: str, log: str, start_timeout: float = 600.0, env: Optional[dict] = None):
        self.url = url
        self.logf = open(log, "w")
        self.p = subprocess.Popen(shlex.split(cmd), stdout=self.logf, stderr=subprocess.STDOUT,
                                  start_new_session=True, env=dict(os.environ, **(env or {})))
        t_end = time.time() + start_timeout
        while time.time() < t_end:
            if self.p.poll() is not None:
                self.logf.close()
                raise RuntimeError(f"server exited with {self.p.returncode} (log: {log})")
            try:
                if json.loads(_client.get(url.rstrip("/") + "/health", 2.0)).get("ok"):
                    return
            except Exception:  # noqa: BLE001  (not up yet)
                pass
            time.sleep(1.0)
        self.stop()
        raise RuntimeError(f"server did not come up in {start_timeout:.0f} s (log: {log})")

    def stop(self) -> dict:
        rc, killed = self.p.poll(), False
        if rc is None:
            os.killpg(self.p.pid, signal.SIGTERM)
            try:
                rc = self.p.wait(timeout=60)
            except subprocess.TimeoutExpired:
                killed = True
                os.killpg(self.p.pid, signal.SIGKILL)
                rc = self.p.wait(timeout=30)
        if not self.logf.closed:
            self.logf.close()
        return {"exit_code": rc, "killed": killed}


def _write(path: str, obj) -> None:
    with open(path, "w") as f:
        json.dump(obj, f, indent=1, default=str)


def run_one(name: str, args: str, out: str, serve_cmd: str = SERVE_CMD, reference: Optional[dict] = None,
            noise: Optional[dict] = None, probes: Optional[dict] = None, start_timeout: float = 600.0,
            env: Optional[dict] = None) -> dict:
    """Serve one stack and probe it; every result is written to out/runs/NAME/ and returned."""
    probes = probes or {}
    d = os.path.join(out, "runs", name)
    os.makedirs(d, exist_ok=True)
    port = free_port()
    url = f"http://127.0.0.1:{port}"
    alerts = os.path.join(d, "alerts.jsonl")
    open(alerts, "w").close()
    cmd = f"{serve_cmd} {args} --port {port} --alerts {shlex.quote(alerts)}"
    res: dict = {"name": name, "args": args, "command": cmd, "url": url, "dir": d}
    t0 = time.time()
    srv = Server(cmd, url, os.path.join(d, "server.log"), start_timeout, env)
    try:
        res["ready"] = ready.check(url, probe=True)
        if reference is None:
            res["quality_reference"] = gate_model.reference_url(url, **probes.get("quality", {}))
        else:
            res["quality"] = gate_model.check_url(reference, url, noise)
        if not probes.get("no_perf"):
            res["perf"] = perf.measure(url, **probes.get("perf", {}))
        if not probes.get("no_isolation"):
            res["isolation"] = isolation.run(url, **probes.get("isolation", {}))
        if not probes.get("no_consistency"):
            res["consistency"] = consistency.run(url, **probes.get("consistency", {}))
        res["metrics"] = _client.get(url.rstrip("/") + "/metrics")
        res["stack"] = ready._stack(_client.parse_metrics(res["metrics"]))
    finally:
        res["server_stop"] = srv.stop()
        res["seconds"] = round(time.time() - t0, 1)
    for k in ("ready", "quality_reference", "quality", "perf", "isolation", "consistency"):
        if k in res:
            _write(os.path.join(d, f"{k}.json"), res[k])
    with open(os.path.join(d, "metrics.txt"), "w") as f:
        f.write(res["metrics"])
    res["alerts"] = decide.read_alerts(alerts)
    return res


def tested_conditions(base: dict, probes: dict) -> dict:
    """What the qualification exercised: the server arguments, the longest prompt and the load."""
    longest = 0
    for r in (base,):
        m = _client.parse_metrics(r.get("metrics", ""))
        longest = max(longest, int(m.get("sdcguard_longest_prompt_tokens", 0)))
    pl = (base.get("perf") or {}).get("load") or {}
    return {"longest_prompt": longest, "max_tokens": pl.get("max_tokens"), "concurrency": pl.get("concurrency"),
            "perf_prompts": pl.get("prompts"), "quality": probes.get("quality", {})}


def set_aside_earlier(out: str) -> Optional[str]:
    names = [n for n in os.listdir(out) if n.startswith(("decision_", "repro_")) or n in
             ("report.txt", "tested_conditions.json", "runs")]
    if not names:
        return None
    dest = os.path.join(out, time.strftime("earlier-%Y%m%d-%H%M%S"))
    os.makedirs(dest)
    for n in names:
        os.replace(os.path.join(out, n), os.path.join(dest, n))
    return dest


def write_repro(out: str, name: str, baseline: str, args: str, a) -> str:
    p = os.path.join(out, f"repro_{name}.sh")
    cmd = [sys.executable, "-m", "sdcguard_b200.tools.qualify", "--out", os.path.join(out, f"repro-{name}"),
           "--serve-cmd", a.serve_cmd, "--baseline", baseline, "--candidate", f"{name}={args}",
           "--concurrency", str(a.concurrency), "--max-tokens", str(a.max_tokens), "--rounds", str(a.rounds)]
    if a.policy:
        cmd += ["--policy", os.path.abspath(a.policy)]
    for flag in ("no_perf", "no_isolation", "no_consistency"):
        if getattr(a, flag):
            cmd.append("--" + flag.replace("_", "-"))
    with open(p, "w") as f:
        f.write("#!/bin/sh\n# rerun the qualification of one candidate against the same baseline\nset -e\n"
                + " ".join(shlex.quote(c) for c in cmd) + "\n")
    os.chmod(p, 0o755)
    return p


def decide_one(cand: dict, base: dict, policy: Optional[dict], tested: dict) -> dict:
    d = decide.decide(policy, quality=cand.get("quality"), alerts=cand["alerts"], metrics=[cand["metrics"]],
                      perf_before=base.get("perf"), perf_after=cand.get("perf"), isolation_run=cand.get("isolation"),
                      consistency_run=cand.get("consistency"), consistency_baseline=base.get("consistency"),
                      baseline_stack=base.get("stack"))
    d["tested"] = tested
    d["candidate"] = {"name": cand["name"], "args": cand["args"]}
    return d


def report(rows: list) -> str:
    lines = ["qualification report", ""]
    head = f"{'candidate':20s} {'decision':12s} {'arithmetic':18s} {'approximation':14s} {'perf':10s} " \
           f"{'isolation':13s} {'consistency':12s}"
    lines.append(head)
    for name, d in rows:
        tp = ((d["performance"].get("metrics") or {}).get("output_tokens_per_s") or {}).get("change")
        lines.append(f"{name:20s} {d['decision']:12s} {d['arithmetic']['verdict']:18s} "
                     f"{d['approximation']['verdict']:14s} {(f'{tp:+.1%}' if tp is not None else '-'):10s} "
                     f"{d['isolation']['verdict']:13s} {d['consistency']['verdict']:12s}")
    for name, d in rows:
        lines += ["", f"== {name}", decide.render(d)]
    return "\n".join(lines) + "\n"


def _pairs(items: list) -> list:
    out = []
    for i, it in enumerate(items):
        name, sep, args = it.partition("=")
        if not sep or " " in name or not name:
            name, args = f"candidate{i + 1}", it
        out.append((name, args))
    if len({n for n, _ in out}) != len(out):
        raise ValueError("candidate names must differ")
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="sdcguard qualify", description=__doc__.split("\n\n")[0])
    ap.add_argument("--out", required=True)
    ap.add_argument("--baseline", required=True, help="server arguments of the trusted stack")
    ap.add_argument("--candidate", action="append", required=True, help="[NAME=]server arguments (repeat)")
    ap.add_argument("--serve-cmd", default=SERVE_CMD)
    ap.add_argument("--policy")
    ap.add_argument("--repeat-baseline", dest="repeat", action="store_true", default=True)
    ap.add_argument("--no-repeat-baseline", dest="repeat", action="store_false")
    ap.add_argument("--no-perf", action="store_true")
    ap.add_argument("--no-isolation", action="store_true")
    ap.add_argument("--no-consistency", action="store_true")
    ap.add_argument("--concurrency", type=int, default=8)
    ap.add_argument("--max-tokens", type=int, default=32)
    ap.add_argument("--rounds", type=int, default=3)
    ap.add_argument("--prompts-file")
    ap.add_argument("--quality-prompts", type=int, default=8)
    ap.add_argument("--startup-timeout", type=float, default=600.0)
    ap.add_argument("--env", action="append", default=[], help="KEY=VALUE for every server (repeat)")
    a = ap.parse_args(argv)
    os.makedirs(a.out, exist_ok=True)
    moved = set_aside_earlier(a.out)
    if moved:
        print(f"earlier results moved to {moved}")
    cands = _pairs(a.candidate)
    policy = None
    if a.policy:
        with open(a.policy) as f:
            policy = json.load(f)
    decide.policy_with_defaults(policy)                      # a bad policy fails before any server starts
    env = dict(kv.split("=", 1) for kv in a.env)
    probes = {"quality": {"prompts": a.quality_prompts},
              "perf": {"prompts": perf.read_prompts(a.prompts_file) if a.prompts_file else None,
                       "concurrency": a.concurrency, "max_tokens": a.max_tokens, "rounds": a.rounds},
              "no_perf": a.no_perf, "no_isolation": a.no_isolation, "no_consistency": a.no_consistency}
    base = run_one("baseline", a.baseline, a.out, a.serve_cmd, probes=probes, start_timeout=a.startup_timeout,
                   env=env)
    ref = base["quality_reference"]
    noise = None
    if a.repeat:
        again = run_one("baseline-repeat", a.baseline, a.out, a.serve_cmd, reference=ref,
                        probes=dict(probes, no_perf=True, no_isolation=True, no_consistency=True),
                        start_timeout=a.startup_timeout, env=env)
        noise = again["quality"]
    tested = tested_conditions(base, probes)
    _write(os.path.join(a.out, "tested_conditions.json"), tested)
    rows = []
    for name, args in cands:
        try:
            cand = run_one(name, args, a.out, a.serve_cmd, reference=ref, noise=noise, probes=probes,
                           start_timeout=a.startup_timeout, env=env)
            d = decide_one(cand, base, policy, tested)
        except Exception as e:  # noqa: BLE001  (a candidate that cannot be served is recorded, not decided)
            d = decide.decide(policy)
            d.update({"decision": "NOT DECIDED", "why": [f"the candidate could not be qualified: {e}"[:500]],
                      "candidate": {"name": name, "args": args}, "tested": tested})
        _write(os.path.join(a.out, f"decision_{name}.json"), d)
        with open(os.path.join(a.out, f"decision_{name}.txt"), "w") as f:
            f.write(decide.render(d) + "\n")
        write_repro(a.out, name, a.baseline, args, a)
        rows.append((name, d))
    text = report(rows)
    with open(os.path.join(a.out, "report.txt"), "w") as f:
        f.write(text)
    print(text)
    words = [d["decision"] for _, d in rows]
    return 0 if all(w == "ACCEPT" for w in words) else 1 if "REJECT" in words else 2


if __name__ == "__main__":
    raise SystemExit(main())
