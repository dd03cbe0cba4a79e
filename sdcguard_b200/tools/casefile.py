"""Incident casefile for one flagged GEMM block: what its evidence and its replays support, and what they don't.

    case = capture(x, w, y, row, block)           # the flagged row of x, the 128 weight rows of the block, the
    save(case, "case_0.pt")                       # recorded output block, the software stack and the GPU
    python -m sdcguard_b200.tools.casefile case_0.pt --replay-here 50        # replay here, then the casefile
    python -m sdcguard_b200.tools.casefile case_0.pt --replays peer.json    # add replays run on other GPUs
    python -m sdcguard_b200.tools.casefile case_0.pt --save-replay peer.json --replay-here 50   # on a peer

The same alarm can come from a GPU that computed wrong once, a GPU that keeps computing wrong, a library or
configuration defect, or the check itself. The casefile collects the evidence that separates them:

  recheck   the recorded output block against a float64 CPU recomputation of the same inputs: outside the rounding
            envelope (bf16 output rounding plus the fp32 accumulation bound) = the GPU's output was wrong
  replays   the same inputs through this library's checked GEMM (and the library GEMM) on the incident GPU (same
            UUID) and on peers: does the wrong output come back, and with which software stack

and scores each explanation as supported / contradicted / not tested from that evidence only:

  transient fault on the incident GPU   wrong output; same-GPU replays ran and never reproduced it
  persistent defect of the incident GPU wrong output; reproduced on the incident GPU, not on peers with its stack
  software or library defect            reproduced on peers with the incident's stack
  false alarm of the check              the recorded output is within the envelope

The outcome is "most consistent with" an explanation when exactly one is supported and nothing contradicts it,
INCONCLUSIVE otherwise, with the replays that would settle it. A replay counts only for this exact case (SHA-256).
Known cuBLAS issues matching the incident's stack are listed as leads.

Reference: src/sdcguard/casefile.py:1-30 (explanations, evidence rules, outcome wording), `classify_replay` :229.
"""
from __future__ import annotations

import argparse
import hashlib
import io
import json
import math

import torch

from ..utils.events import load_evidence, plain

SUPPORTED, CONTRADICTED, NOT_TESTED = "supported", "contradicted", "not tested"
WEAK = 10           # fewer replays than this on one side are weak evidence of absence


def stack() -> dict:
    import torch as t
    d = {"torch": t.__version__, "cuda": t.version.cuda}
    if t.cuda.is_available():
        p = t.cuda.get_device_properties(t.cuda.current_device())
        d.update(gpu_name=p.name, gpu_uuid=str(getattr(p, "uuid", "")), cc=f"{p.major}.{p.minor}")
    try:
        from .known_issues import cublas_version
        d["cublas"] = cublas_version()
    except Exception:  # noqa: BLE001  (recorded when readable)
        d["cublas"] = None
    return d


def capture(x: torch.Tensor, w: torch.Tensor, y: torch.Tensor, row: int, block: int, note: str = "") -> dict:
    """The evidence of a flagged (row, 128-column block) of y = x @ w^T: host copies of what a recheck needs."""
    c0, c1 = block * 128, min((block + 1) * 128, w.shape[0])
    return {"format": "sdcguard-b200-case/1", "kind": "gemm", "row": row, "block": block, "note": note,
            "x_row": x[row].detach().to("cpu", torch.bfloat16).clone(),
            "w_block": w[c0:c1].detach().to("cpu", torch.bfloat16).clone(),
            "y_block": y[row, c0:c1].detach().to("cpu", torch.bfloat16).clone(), "stack": plain(stack())}


def sha256(case: dict) -> str:
    buf = io.BytesIO()
    torch.save({k: case[k] for k in ("x_row", "w_block", "y_block")}, buf)
    return hashlib.sha256(buf.getvalue()).hexdigest()


def save(case: dict, path: str) -> str:
    torch.save(case, path)
    return sha256(case)


def recheck(case: dict) -> dict:
    """float64 CPU recomputation of the block and the per-element envelope: bf16 rounding of the output (half an
    ulp, at most 2^-8 relative) plus k u |x| . |w| for any fp32 accumulation order."""
    x, w, y = case["x_row"].double(), case["w_block"].double(), case["y_block"].double()
    ref = w @ x
    k = x.numel()
    env = 2.0 ** -8 * ref.abs() + 1.01 * k * 2.0 ** -24 * (w.abs() @ x.abs()) + 1e-30
    dev = (y - ref).abs() / env
    bad = (dev > 1) | ~torch.isfinite(y)
    return {"elements": y.numel(), "outside_envelope": int(bad.sum()), "worst": float(dev.nan_to_num(math.inf).max()),
            "first_bad_column": int(bad.nonzero()[0, 0]) + case["block"] * 128 if bad.any() else None,
            "output_wrong": bool(bad.any())}


def replay(case: dict, runs: int = 20, device: str = "cuda:0") -> dict:
    """Recompute the block `runs` times with this library's checked GEMM (M = 1 row, N = the block) and with the
    library GEMM; count runs whose output differs from the float64 envelope or that alarm."""
    from ..numerics import abft
    from ..ops import gemm
    dev = torch.device(device)
    x = case["x_row"].to(dev).view(1, -1).contiguous()
    w = case["w_block"].to(dev).contiguous()
    k = x.shape[1]
    n = w.shape[0]
    pad = (-n) % 128
    wp = torch.cat([w, torch.zeros(pad, k, dtype=w.dtype, device=dev)]) if pad else w
    cw = gemm.CheckedWeight(wp)
    st = gemm.StateTable(dev, 2)
    slot = st.add("replay", cw.nb)
    ref = case["w_block"].double() @ case["x_row"].double()
    env = 2.0 ** -8 * ref.abs() + 1.01 * k * 2.0 ** -24 * (case["w_block"].double().abs() @ case["x_row"].double().abs())
    wrong_sdc = wrong_lib = alarms = 0
    for _ in range(runs):
        y = gemm.checked_linear(x, cw, st.state, slot)[0, :n].double().cpu()
        wrong_sdc += int(((y - ref).abs() > env + 1e-30).any())
        alarms += int(st.read(reset=True)[0]["z"] > abft.Z_ALARM)
        yl = (x @ w.t())[0].double().cpu()
        wrong_lib += int(((yl - ref).abs() > env + 1e-30).any())
    same = stack()
    return {"case_sha256": sha256(case), "gpu_uuid": same.get("gpu_uuid"), "stack": same, "runs": runs,
            "reproduced_checked_kernel": wrong_sdc, "reproduced_library": wrong_lib, "alarms": alarms,
            "reproduced": wrong_sdc + wrong_lib + alarms > 0}


def _same_stack(a: dict, b: dict) -> bool:
    return all(a.get(k) == b.get(k) for k in ("torch", "cuda", "gpu_name"))


def casefile(case: dict, replays: list[dict]) -> dict:
    h = sha256(case)
    rc = recheck(case)
    inc = case["stack"]
    used = [r for r in replays if r.get("case_sha256") == h]
    ignored = len(replays) - len(used)
    here = [r for r in used if r.get("gpu_uuid") and r["gpu_uuid"] == inc.get("gpu_uuid")]
    peers = [r for r in used if r not in here and _same_stack(r.get("stack", {}), inc)]
    here_runs, here_rep = sum(r["runs"] for r in here), sum(r["reproduced"] for r in here)
    peer_runs, peer_rep = sum(r["runs"] for r in peers), sum(r["reproduced"] for r in peers)
    ex = {}
    wrong = rc["output_wrong"]
    ex["false alarm of the check"] = CONTRADICTED if wrong else SUPPORTED
    if not here:
        ex["transient fault on the incident GPU"] = NOT_TESTED if wrong else CONTRADICTED
        ex["persistent defect of the incident GPU"] = NOT_TESTED if wrong else CONTRADICTED
    else:
        ex["transient fault on the incident GPU"] = (CONTRADICTED if here_rep or not wrong else
                                                     SUPPORTED if here_runs >= WEAK else NOT_TESTED)
        ex["persistent defect of the incident GPU"] = (CONTRADICTED if not wrong or (not here_rep and here_runs >= WEAK)
                                                       or peer_rep else SUPPORTED if here_rep else NOT_TESTED)
    ex["software or library defect"] = (SUPPORTED if peer_rep else CONTRADICTED if peer_runs >= WEAK or not wrong
                                        else NOT_TESTED)
    sup = [k for k, v in ex.items() if v == SUPPORTED]
    outcome = f"most consistent with: {sup[0]}" if len(sup) == 1 else "INCONCLUSIVE"
    nxt = []
    if wrong and here_runs < WEAK:
        nxt.append(f"replay on the incident GPU (at least {WEAK} runs)")
    if wrong and peer_runs < WEAK:
        nxt.append(f"replay on a peer GPU with the same software stack (at least {WEAK} runs)")
    from .known_issues import match
    leads = [{"id": r["id"], "verdict": r["verdict"], "when": r["when"]}
             for r in match({"cublas": inc.get("cublas"), "cc": inc.get("cc")}) if r["verdict"] in ("applies",
                                                                                                  "may apply")]
    return {"case_sha256": h, "location": {"row": case["row"], "block": case["block"]}, "recheck": rc,
            "replays": {"incident_gpu": {"runs": here_runs, "reproduced": here_rep},
                        "peers_same_stack": {"runs": peer_runs, "reproduced": peer_rep},
                        "ignored_other_case": ignored},
            "explanations": ex, "outcome": outcome, "next_steps": nxt, "leads": leads, "stack": inc}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m sdcguard_b200.tools.casefile")
    ap.add_argument("case")
    ap.add_argument("--replays", nargs="*", default=[])
    ap.add_argument("--replay-here", type=int, default=0)
    ap.add_argument("--save-replay")
    ap.add_argument("--device", default="cuda:0")
    a = ap.parse_args(argv)
    case = load_evidence(a.case)
    reps = []
    for p in a.replays:
        with open(p) as f:
            reps.append(json.load(f))
    if a.replay_here:
        r = replay(case, a.replay_here, a.device)
        reps.append(r)
        if a.save_replay:
            with open(a.save_replay, "w") as f:
                json.dump(r, f, indent=1)
    print(json.dumps(casefile(case, reps), indent=1))
    return 0


def replay_main(argv=None) -> int:
    """`sdcguard replay CASE.pt [--times N] [--device D] [--save OUT.json]`: recompute a captured block here, print
    the replay record (the casefile's input), exit 1 when a recomputation came out wrong or alarmed again, 0 when
    none did, 2 when it could not run. (Reference: `sdcguard replay`, src/sdcguard/cli.py:214, screen.py:657.)"""
    ap = argparse.ArgumentParser(prog="sdcguard replay")
    ap.add_argument("case")
    ap.add_argument("--times", type=int, default=200)
    ap.add_argument("--device", default="cuda:0")
    ap.add_argument("--save")
    a = ap.parse_args(argv)
    if a.times < 1:
        print("sdcguard replay: --times must be at least 1")
        return 2
    try:
        case = load_evidence(a.case)
        r = replay(case, a.times, a.device)
    except (OSError, RuntimeError, KeyError, ValueError) as e:
        print(f"sdcguard replay: could not run ({type(e).__name__}: {e})")
        return 2
    print(json.dumps(r, indent=1, default=str))
    if a.save:
        with open(a.save, "w") as f:
            json.dump(r, f, indent=1, default=str)
    return 1 if r["reproduced"] else 0


if __name__ == "__main__":
    raise SystemExit(main())
