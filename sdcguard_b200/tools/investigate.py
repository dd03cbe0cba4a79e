"""Investigate a flagged GEMM case: does the wrong result follow a GPU, or the software path?

    python -m sdcguard_b200.tools.investigate case_0.pt [--runs 20]

Replays the case (`casefile.replay`) on every GPU visible here, through this library's checked tcgen05 GEMM and
through the library GEMM, and changes one thing at a time:

  DEVICE          wrong on some GPUs and right on the others, with the same software: drain that GPU, keep the case
                  for an RMA
  SOFTWARE PATH   wrong on every GPU through one path and right through the other: pin or change the path; moving
                  the job will not fix it
  NOT ONE GPU     wrong on every one of two or more GPUs through both paths
  NOT REPRODUCED  right everywhere: a transient fault, or one that needs the original conditions
  INCONCLUSIVE    one GPU only and it reproduced (one GPU cannot tell a device from the software), or a replay failed

Reference: src/sdcguard/investigate.py:1-25 (factors and verdict words).
"""
from __future__ import annotations

import argparse
import json

import torch

from ..utils.events import load_evidence

from .casefile import replay


def investigate(case: dict, runs: int = 20, devices=None) -> dict:
    devices = devices if devices is not None else [f"cuda:{i}" for i in range(torch.cuda.device_count())]
    rows, errors = [], []
    for d in devices:
        try:
            r = replay(case, runs, d)
            rows.append({"device": d, "gpu_uuid": r["gpu_uuid"], "checked_kernel_wrong": r["reproduced_checked_kernel"],
                         "library_wrong": r["reproduced_library"], "alarms": r["alarms"]})
        except Exception as e:  # noqa: BLE001  (reported)
            errors.append({"device": d, "error": f"{type(e).__name__}: {e}"})
    return {"devices": rows, "errors": errors, "runs": runs, "verdict": classify(rows, errors)}


def classify(rows: list[dict], errors: list) -> str:
    if errors or not rows:
        return "INCONCLUSIVE"
    bad = [r for r in rows if r["checked_kernel_wrong"] or r["library_wrong"] or r["alarms"]]
    if not bad:
        return "NOT REPRODUCED"
    if len(rows) == 1:
        return "INCONCLUSIVE"
    if len(bad) < len(rows):
        return "DEVICE"
    ours = all(r["checked_kernel_wrong"] or r["alarms"] for r in rows)
    lib = all(r["library_wrong"] for r in rows)
    if ours != lib:
        return "SOFTWARE PATH"
    return "NOT ONE GPU"


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m sdcguard_b200.tools.investigate")
    ap.add_argument("case")
    ap.add_argument("--runs", type=int, default=20)
    a = ap.parse_args(argv)
    r = investigate(load_evidence(a.case), a.runs)
    print(json.dumps(r, indent=1))
    return 0 if r["verdict"] == "NOT REPRODUCED" else 1


if __name__ == "__main__":
    raise SystemExit(main())
