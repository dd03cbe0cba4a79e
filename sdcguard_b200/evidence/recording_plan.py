"""Prepare the instructions for a passive recording of a prefill/decode deployment of this engine, without starting
anything: which command each worker runs with which recording options, where the files go, and how they are judged
afterwards.

    python -m sdcguard_b200.evidence.recording_plan DEPLOYMENT.json --out PLAN.json [--dir rec/]
    sdcguard record-plan DEPLOYMENT.json --out PLAN.json

The deployment is validated with the static contracts first (`evidence.config`); a deployment whose contracts are
violated gets no plan (recording a configuration that is already known to be unsafe proves nothing). The plan names,
per decode worker, the recording directory (REQUEST_PLAN.json, OBSERVER.json, CACHE.json,
CACHED_PREFIX_VERIFICATION.json, RESULT.json and lifetime.jsonl, as `serve.pd_mp` writes them), the environment
(`SDCGUARD_SIGN_SEED` pinned so replays reproduce the sign pattern), and the offline steps that judge it: `sdcguard
gate`, `sdcguard assess`, `sdcguard assignment`, `sdcguard forward-inputs`, `sdcguard evidence build`.

Reference: src/sdcguard/recording_plan.py:1-10 (`validate_deployment`, `environment_snippet`,
`prepare_recording_plan`).
"""
from __future__ import annotations

import argparse
import json
import os
import shlex
import sys

from . import config

SCHEMA = "sdcguard_b200.recording-plan.v1"


def validate_deployment(doc: dict, prov: dict) -> tuple[bool, dict]:
    a = config.assess(doc, prov)
    return a["verdict"] != "FAIL", a


def environment_snippet(seed: int = 1) -> dict:
    return {"SDCGUARD_SIGN_SEED": str(seed), "NCCL_DEBUG": "WARN", "MASTER_ADDR": "127.0.0.1"}


def prepare_recording_plan(doc: dict, prov: dict, out_dir: str = "rec", seed: int = 1) -> dict:
    ok, assessment = validate_deployment(doc, prov)
    if not ok:
        raise ValueError("the deployment violates its static contracts: "
                         + "; ".join(r["id"] for w in assessment["workers"] for r in w["rules"]
                                     if r["verdict"] == "violated"))
    ws = doc["workers"]
    P = sum(1 for w in ws if w.get("role") == "prefill")
    D = sum(1 for w in ws if w.get("role") == "decode")
    if P < 1 or D < 1:
        raise ValueError("a prefill/decode recording needs at least one prefill and one decode worker")
    verify = all(w.get("verify_cached_prefix") is True for w in ws if w.get("role") == "decode")
    env = environment_snippet(seed)
    cmd = (["torchrun", "--nnodes=1", f"--nproc-per-node={P + D}", "--master-addr", "127.0.0.1",
            "-m", "sdcguard_b200.serve.pd_mp", "--prefill", str(P), "--model", str(doc["model"].get("name")),
            "--out", out_dir] + (["--verify-cached-prefix"] if verify else []))
    judge = []
    for c in range(D):
        d = os.path.join(out_dir, f"decode{c}")
        ev = os.path.join(d, "lifetime.jsonl")
        judge += [["sdcguard", "gate", d],
                  ["sdcguard", "assess", d, "--events", ev, "--json"],
                  ["sdcguard", "assignment", "inspect", ev],
                  ["sdcguard", "forward-inputs", "inspect", ev]]
    return {"schema": SCHEMA, "deployment_binding": prov["binding"], "contracts_verdict": assessment["verdict"],
            "environment": env, "launch": cmd, "launch_shell": " ".join(f"{k}={shlex.quote(v)}" for k, v in env.items())
            + " " + " ".join(shlex.quote(x) for x in cmd),
            "recordings": [os.path.join(out_dir, f"decode{c}") for c in range(D)], "judge": judge,
            "notes": ["the plan starts nothing; the operator runs the launch line",
                      "recordings are passive: the same kernels run with or without them"]}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="sdcguard record-plan")
    ap.add_argument("deployment")
    ap.add_argument("--out", required=True)
    ap.add_argument("--dir", default="rec")
    ap.add_argument("--seed", type=int, default=1)
    a = ap.parse_args(argv)
    try:
        doc, prov = config.load_deployment(a.deployment)
        plan = prepare_recording_plan(doc, prov, a.dir, a.seed)
    except (OSError, ValueError) as e:
        print(f"record-plan: {e}", file=sys.stderr)
        return 2
    with open(a.out, "w") as f:
        json.dump(plan, f, indent=1)
    print(plan["launch_shell"])
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
