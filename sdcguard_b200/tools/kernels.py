"""Which library matmul kernels a workload runs, read from cuBLASLt's own log, and how many of them a test ran.

cuBLAS picks a kernel per call from the shape, the types, the GPU and the process's conditions (an MPS client below
100% gets other kernels), and a library defect can sit in one kernel only; a test proves nothing about kernels it
never ran. With CUBLASLT_LOG_LEVEL=5 cuBLASLt writes one Trace line per matmul call with its descriptors and the
exact kernel configuration (algorithm, tile, stages, split-K, reduction scheme, custom option, cluster shape). This
turns those lines into an inventory and compares inventories:

    python -m sdcguard_b200.tools.kernels record --out serve.json -- python -m sdcguard_b200.serve.tp_serve ...
    python -m sdcguard_b200.tools.kernels coverage serve.json --test screen.json
    python -m sdcguard_b200.tools.kernels diff before.json after.json
    python -m sdcguard_b200.tools.kernels show serve.json
    python -m sdcguard_b200.tools.kernels parse cublaslt.log --out inv.json
    python -m sdcguard_b200.tools.kernels test serve.json --out tested.json [--repeats 3]

An inventory lists each distinct kernel (types, compute type, epilogue, configuration) with its calls, the shapes it
ran and its share of the matmul work (2 m n k batch per call). Coverage counts a workload kernel as exercised when
the test ran the same configuration on the same types (and, strictly, the same shape), weighted by work, and marks
kernels whose configuration matches a listed wrong-result issue (algorithm 66 with split-K, clusters of 4+ CTAs).
This library's checked paths run no cuBLAS at all; the inventory is for unchecked arms and foreign jobs. Lines that
are not matmul Trace lines are ignored; unreadable matmul Trace lines are counted, never guessed.

`test` runs every inventoried call again on this GPU, at its shape, in a fresh process with cuBLASLt's log on: the
operands laid out as the call had them (transposes and batch), random inputs, outputs into NaN-filled buffers, each
shape `--repeats` times, every output judged against float64 with a rounding bound (bf16 / fp16 output rounding plus
fp32 accumulation with tensor-core truncation over k). Per call: PASSED when every run was right and cuBLASLt ran
the same kernel here (the inventory's key among the keys logged for that shape); WRONG when an output element was
outside the bound or never written; OTHER KERNEL when the runs were right but cuBLASLt chose another kernel here
(other conditions: run it where the workload runs); NOT RUN for calls this cannot replay (types other than bf16 /
fp16 in and out with fp32 compute, epilogues other than the default, outputs too large for the float64 check).
Random inputs: a fault that needs the workload's own data or memory layout may not show.

Reference: src/sdcguard/kernels.py:1-44 (commands, keys and coverage rules), `parse_line` :82, `test_calls` :346,
`main` :522.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import subprocess
import sys
import tempfile
from typing import Iterable, Optional

FORMAT = "sdcguard-b200-kernels/1"
_TRACE = re.compile(r"\[Trace\]\[(cublasLt\w*Matmul)\]\s?(.*)$")
_TOKEN = re.compile(r"(\w+)=(\[[^\]]*\]|\S+)")
_KV = re.compile(r"(\w+)=([^\s\]]+)")
_STRIP = ("MATMUL_TILE_", "MATMUL_STAGES_", "CLUSTER_SHAPE_", "REDUCTION_SCHEME_", "CUBLASLT_", "EPILOGUE_")
KERNEL_FIELDS = ("algoId", "tile", "stages", "numSplitsK", "reductionScheme", "customOption", "clusterShape",
                 "swizzle", "innerShape")
TYPE_NAMES = {"R_16F": "fp16", "R_16BF": "bf16", "R_32F": "fp32", "R_64F": "fp64", "R_8F_E4M3": "fp8e4m3",
              "R_8F_E5M2": "fp8e5m2", "R_8I": "int8", "R_32I": "int32", "R_4F_E2M1": "fp4e2m1"}


def _clean(v: str) -> str:
    for p in _STRIP:
        if v.startswith(p):
            return v[len(p):]
    return v


def _group(text: str) -> dict:
    return {k: _clean(v) for k, v in _KV.findall(text[1:-1])}


def parse_line(line: str) -> Optional[dict]:
    """A cuBLASLt matmul Trace line as a call dict; None for other lines; ValueError for a matmul Trace line that
    lacks A / D descriptors or the kernel configuration."""
    mt = _TRACE.search(line)
    if not mt:
        return None
    fn, rest = mt.groups()
    f = {k: (_group(v) if v.startswith("[") else v) for k, v in _TOKEN.findall(rest)}
    a, d, algo = f.get("Adesc"), f.get("Ddesc"), f.get("algo")
    if not (isinstance(a, dict) and isinstance(d, dict) and isinstance(algo, dict) and "algoId" in algo):
        raise ValueError("matmul Trace line without A / D descriptors or kernel configuration")
    comp = f["computeDesc"] if isinstance(f.get("computeDesc"), dict) else {}
    b = f["Bdesc"] if isinstance(f.get("Bdesc"), dict) else {}
    c = f["Cdesc"] if isinstance(f.get("Cdesc"), dict) else {}
    try:
        m, n = int(d["rows"]), int(d["cols"])
        k = int(a["rows"] if comp.get("transa", "OP_N") == "OP_T" else a["cols"])
    except (KeyError, ValueError) as e:
        raise ValueError(f"matmul Trace line with unreadable dimensions ({e})") from None
    batch = max([1] + [int(x["batchCount"]) for x in (a, d) if str(x.get("batchCount", "")).isdigit()])
    return {"fn": fn, "m": m, "n": n, "k": k, "batch": batch,
            "types": [TYPE_NAMES.get(x.get("type", "?"), x.get("type", "?")) for x in (a, b, c, d)],
            "transa": comp.get("transa", "OP_N"), "transb": comp.get("transb", "OP_N"),
            "ld": [a.get("ld"), b.get("ld"), d.get("ld")], "compute": comp.get("computeType", "?"),
            "epilogue": comp.get("epilogue", "DEFAULT"), "sm_count_target": comp.get("smCountTarget"),
            "algo": algo}


def kernel_key(c: dict) -> str:
    algo = c["algo"]
    cfg = [f"{k}={algo[k]}" for k in KERNEL_FIELDS if k in algo]
    cfg += [f"{k}={algo[k]}" for k in sorted(algo) if k not in KERNEL_FIELDS]
    t = c["types"]
    return f"{t[0]}x{t[1]}->{t[3]} compute={c['compute']} epilogue={c['epilogue']} {c['fn']} " + " ".join(cfg)


def shape_key(c: dict) -> str:
    return (f"m={c['m']} n={c['n']} k={c['k']} batch={c['batch']} {c['transa']}/{c['transb']} "
            f"ld={','.join(str(x) for x in c['ld'])}" + (f" sms={c['sm_count_target']}" if c['sm_count_target'] else ""))


def issue_flags(algo: dict) -> list[str]:
    """Configurations named by listed wrong-result issues (tools/data/cublas_issues.json)."""
    flags = []
    if algo.get("algoId") == "66":
        cs = algo.get("clusterShape", "")
        dims = [int(x) for x in re.findall(r"\d+", cs)]
        if dims and dims[0] * (dims[1] if len(dims) > 1 else 1) >= 4:
            flags.append("6862950 (cluster of 4+ CTAs, Hopper under MPS)")
        if algo.get("numSplitsK", "1") not in ("0", "1"):
            flags.append("6580689 (split-K)")
    return flags


def inventory(lines: Iterable[str], source: str = "") -> dict:
    kernels: dict = {}
    calls = unreadable = 0
    for line in lines:
        try:
            c = parse_line(line)
        except ValueError:
            unreadable += 1
            continue
        if c is None:
            continue
        calls += 1
        key = kernel_key(c)
        work = 2 * c["m"] * c["n"] * c["k"] * c["batch"]
        e = kernels.setdefault(key, {"calls": 0, "work": 0, "shapes": {}, "types": c["types"], "algo": c["algo"],
                                     "flags": issue_flags(c["algo"])})
        e["calls"] += 1
        e["work"] += work
        sk = shape_key(c)
        e["shapes"][sk] = e["shapes"].get(sk, 0) + 1
    total = sum(e["work"] for e in kernels.values()) or 1
    for e in kernels.values():
        e["work_share"] = round(e["work"] / total, 6)
    return {"format": FORMAT, "source": source, "calls": calls, "unreadable_lines": unreadable,
            "kernels": dict(sorted(kernels.items(), key=lambda kv: -kv[1]["work"]))}


def coverage(workload: dict, tests: list[dict]) -> dict:
    """Share of the workload's kernels (by count and by work) that some test ran: same kernel, and same kernel on
    the same shape."""
    tk = {}
    for t in tests:
        for key, e in t["kernels"].items():
            tk.setdefault(key, set()).update(e["shapes"])
    rows, w_k, w_s, n_k = [], 0.0, 0.0, 0
    for key, e in workload["kernels"].items():
        ran = key in tk
        same = sum(1 for s in e["shapes"] if ran and s in tk[key])
        w_k += e["work_share"] if ran else 0
        w_s += e["work_share"] * (same / len(e["shapes"])) if ran else 0
        n_k += ran
        rows.append({"kernel": key, "work_share": e["work_share"], "exercised": ran,
                     "shapes_exercised": f"{same}/{len(e['shapes'])}", "flags": e["flags"]})
    n = len(workload["kernels"])
    return {"kernels": n, "kernels_exercised": n_k, "work_exercised": round(w_k, 4),
            "work_exercised_same_shape": round(w_s, 4), "not_exercised": [r for r in rows if not r["exercised"]],
            "flagged": [r for r in rows if r["flags"]], "rows": rows}


def diff(a: dict, b: dict) -> dict:
    ka, kb = set(a["kernels"]), set(b["kernels"])
    return {"only_before": sorted(ka - kb), "only_after": sorted(kb - ka), "both": len(ka & kb),
            "work_moved": round(sum(b["kernels"][k]["work_share"] for k in kb - ka), 4)}


def record(cmd: list[str], out: str, seconds: Optional[float] = None) -> dict:
    """Run cmd with cuBLASLt logging into a temporary file, then build the inventory."""
    with tempfile.TemporaryDirectory() as d:
        log = os.path.join(d, "cublaslt.log")
        env = dict(os.environ, CUBLASLT_LOG_LEVEL="5", CUBLASLT_LOG_FILE=log)
        p = subprocess.Popen(cmd, env=env)
        try:
            p.wait(timeout=seconds)
        except subprocess.TimeoutExpired:
            p.terminate()
            p.wait(timeout=60)
        files = [os.path.join(d, f) for f in os.listdir(d)]
        lines = []
        for f in files:
            with open(f, errors="replace") as fh:
                lines.extend(fh)
    inv = inventory(lines, source=" ".join(cmd))
    inv["exit_code"] = p.returncode
    with open(out, "w") as f:
        json.dump(inv, f, indent=1)
    return inv


_SHAPE = re.compile(r"m=(\d+) n=(\d+) k=(\d+) batch=(\d+) (OP_\w)/(OP_\w)")
REPLAY_TYPES = ("bf16", "fp16")
MAX_ELEMENTS = 64e6


def parse_shape(key: str) -> Optional[dict]:
    mt = _SHAPE.match(key)
    if not mt:
        return None
    m, n, k, b, ta, tb = mt.groups()
    return {"m": int(m), "n": int(n), "k": int(k), "batch": int(b), "transa": ta, "transb": tb}


def rerunnable(e: dict, shape: Optional[dict], max_elements: float = MAX_ELEMENTS) -> Optional[str]:
    """Why an inventoried call cannot be replayed here (None when it can)."""
    t = e["types"]
    if shape is None:
        return "unreadable shape"
    if t[0] not in REPLAY_TYPES or len(set(t[:2] + t[3:])) != 1:
        return f"types {t[0]} x {t[1]} -> {t[3]} (replayed: bf16 or fp16 in and out)"
    if shape["m"] * shape["n"] * shape["batch"] > max_elements:
        return "an output too large for the float64 reference here"
    return None


def _replay_key(e: dict, s: dict) -> tuple:
    return (s["m"], s["n"], s["k"], s["batch"], s["transa"], s["transb"], e["types"][0])


def judge_output(y, ref, a_abs, b_abs, k: int, dtype: str) -> dict:
    """Elements outside |y - ref| <= u_out |ref| + k 2^-22 (|A| |B|) (+ tiny), and elements never written (NaN)."""
    import torch
    u_out = 2.0 ** -8 if dtype == "bf16" else 2.0 ** -11
    mag = torch.matmul(a_abs, b_abs)
    bound = u_out * ref.abs() + k * 2.0 ** -22 * mag + 1e-30
    yd = y.double()
    unwritten = int(torch.isnan(yd).sum())
    bad = int(((yd - ref).abs() > bound).sum()) if not unwritten else int((~torch.isfinite(yd)).sum())
    return {"wrong": bad, "unwritten": unwritten}


def _worker_main(todo_path: str, out_path: str) -> None:
    """Child process of `test`: replays each shape with the operand layouts of its cuBLAS call."""
    import torch
    with open(todo_path) as f:
        todo = json.load(f)
    dev = torch.device("cuda")
    res = []
    for t in todo:
        dt = torch.bfloat16 if t["dtype"] == "bf16" else torch.float16
        m, n, k, b = t["m"], t["n"], t["k"], t["batch"]
        g = torch.Generator(device=dev).manual_seed(1234 + len(res))
        wrong = unwritten = 0
        for _ in range(t["repeats"]):
            # column-major D (m x n) = op(A) op(B) is row-major Y (n x m) = op(B)^T op(A)^T; build each operand in
            # the storage its transpose flag implies so that cuBLAS sees the same call
            A = torch.randn(b, *((m, k) if t["transa"] == "OP_T" else (k, m)), generator=g, device=dev).to(dt)
            B = torch.randn(b, *((k, n) if t["transb"] == "OP_T" else (n, k)), generator=g, device=dev).to(dt)
            a_op = A.transpose(1, 2) if t["transa"] == "OP_T" else A          # (b, k, m) view
            b_op = B.transpose(1, 2) if t["transb"] == "OP_T" else B          # (b, n, k) view
            y = torch.full((b, n, m), float("nan"), dtype=dt, device=dev)
            if b == 1:
                torch.matmul(b_op[0], a_op[0], out=y[0])
            else:
                torch.bmm(b_op, a_op, out=y)
            torch.cuda.synchronize()
            ref = torch.matmul(b_op.double(), a_op.double())
            j = judge_output(y, ref, b_op.double().abs(), a_op.double().abs(), k, t["dtype"])
            wrong += j["wrong"] > 0 or j["unwritten"] > 0
            unwritten += j["unwritten"] > 0
        res.append({"runs": t["repeats"], "runs_wrong": wrong, "runs_unwritten": unwritten})
    with open(out_path, "w") as f:
        json.dump({"results": res, "gpu": torch.cuda.get_device_name(dev)}, f)


def _run_worker(todo: list, log_dir: str, timeout: float = 1800.0) -> tuple:
    os.makedirs(log_dir, exist_ok=True)
    tp, op = os.path.join(log_dir, "todo.json"), os.path.join(log_dir, "results.json")
    log = os.path.join(log_dir, "cublaslt.log")
    with open(tp, "w") as f:
        json.dump(todo, f)
    env = dict(os.environ, CUBLASLT_LOG_LEVEL="5", CUBLASLT_LOG_FILE=log)
    subprocess.run([sys.executable, "-m", "sdcguard_b200.tools.kernels", "_worker", tp, op], env=env, check=True,
                   timeout=timeout)
    with open(op) as f:
        out = json.load(f)
    lines = []
    for name in sorted(os.listdir(log_dir)):
        if name.startswith("cublaslt"):
            with open(os.path.join(log_dir, name), errors="replace") as f:
                lines.extend(f)
    return out, lines


def test_calls(inv: dict, repeats: int = 3, log_dir: str = "kernel_test_logs", max_shapes: int = 200,
               runner=None, max_elements: float = MAX_ELEMENTS) -> dict:
    """The verdict of every inventoried call replayed here (see the module docstring)."""
    todo, index, rows, not_run = [], {}, [], []
    order = sorted(inv["kernels"].items(), key=lambda kv: -kv[1]["work"])
    for key, e in order:
        for sk in e["shapes"]:
            s = parse_shape(sk)
            why = rerunnable(e, s, max_elements)
            if why is None and s is not None:
                rk = _replay_key(e, s)
                if rk not in index:
                    if len(todo) >= max_shapes:
                        why = f"past --max-shapes {max_shapes}"
                    else:
                        index[rk] = len(todo)
                        todo.append(dict(s, dtype=e["types"][0], repeats=repeats))
            rows.append({"kernel": key, "shape": sk, "call": f"{key} | {sk}", "calls_in_workload": e["shapes"][sk],
                         "why_not_run": why, "replay": index.get(_replay_key(e, s)) if s and why is None else None})
    out, lines = (runner or _run_worker)(todo, log_dir) if todo else ({"results": [], "gpu": None}, [])
    ran: dict = {}
    for line in lines:
        try:
            c = parse_line(line)
        except ValueError:
            continue
        if c is None:
            continue
        rk = (c["m"], c["n"], c["k"], c["batch"], c["transa"], c["transb"], c["types"][0])
        ran.setdefault(rk, set()).add(kernel_key(c))
    counts = dict.fromkeys(("PASSED", "WRONG", "OTHER KERNEL", "NOT RUN"), 0)
    calls = []
    for r in rows:
        if r["why_not_run"] is not None:
            counts["NOT RUN"] += 1
            calls.append({"call": r["call"], "kernel": r["kernel"], "verdict": "NOT RUN", "why": r["why_not_run"]})
            continue
        res = out["results"][r["replay"]]
        t = todo[r["replay"]]
        here = ran.get((t["m"], t["n"], t["k"], t["batch"], t["transa"], t["transb"], t["dtype"]), set())
        if res["runs_wrong"]:
            v = "WRONG"
        elif r["kernel"] in here:
            v = "PASSED"
        else:
            v = "OTHER KERNEL"
        counts[v] += 1
        calls.append({"call": r["call"], "kernel": r["kernel"], "verdict": v, "runs": res["runs"],
                      "runs_wrong": res["runs_wrong"], "ran_here": sorted(here)[:4]})
    return {"format": "sdcguard-b200-kernel-test/1", "source": inv.get("source"), "gpu": out.get("gpu"),
            "repeats": repeats, "counts": counts, "calls": calls, "shapes_replayed": len(todo)}


def _load(p: str) -> dict:
    with open(p) as f:
        d = json.load(f)
    if d.get("format") != FORMAT:
        raise SystemExit(f"{p}: not a kernel inventory ({FORMAT})")
    return d


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m sdcguard_b200.tools.kernels")
    sub = ap.add_subparsers(dest="cmd", required=True)
    r = sub.add_parser("record")
    r.add_argument("--out", required=True)
    r.add_argument("--seconds", type=float)
    r.add_argument("command", nargs=argparse.REMAINDER)
    pa = sub.add_parser("parse")
    pa.add_argument("logs", nargs="+")
    pa.add_argument("--out")
    cv = sub.add_parser("coverage")
    cv.add_argument("workload")
    cv.add_argument("--test", nargs="+", required=True)
    df = sub.add_parser("diff")
    df.add_argument("before")
    df.add_argument("after")
    sh = sub.add_parser("show")
    sh.add_argument("inventory")
    te = sub.add_parser("test")
    te.add_argument("inventory")
    te.add_argument("--out")
    te.add_argument("--repeats", type=int, default=3)
    te.add_argument("--max-shapes", type=int, default=200)
    te.add_argument("--log-dir", default="kernel_test_logs")
    wk = sub.add_parser("_worker")
    wk.add_argument("todo")
    wk.add_argument("result")
    a = ap.parse_args(argv)
    if a.cmd == "_worker":
        _worker_main(a.todo, a.result)
        return 0
    if a.cmd == "test":
        r = test_calls(_load(a.inventory), a.repeats, a.log_dir, a.max_shapes)
        if a.out:
            with open(a.out, "w") as f:
                json.dump(r, f, indent=1)
        print(json.dumps(r["counts"]))
        return 1 if r["counts"]["WRONG"] else 0 if r["counts"]["PASSED"] else 2
    if a.cmd == "record":
        cmd = a.command[1:] if a.command[:1] == ["--"] else a.command
        inv = record(cmd, a.out, a.seconds)
        print(json.dumps({"calls": inv["calls"], "kernels": len(inv["kernels"]), "out": a.out}))
    elif a.cmd == "parse":
        lines = []
        for p in a.logs:
            with open(p, errors="replace") as f:
                lines.extend(f)
        inv = inventory(lines, source=",".join(a.logs))
        text = json.dumps(inv, indent=1)
        if a.out:
            with open(a.out, "w") as f:
                f.write(text)
        else:
            print(text)
    elif a.cmd == "coverage":
        c = coverage(_load(a.workload), [_load(t) for t in a.test])
        print(json.dumps({k: v for k, v in c.items() if k != "rows"}, indent=1))
        return 0 if not c["not_exercised"] else 2
    elif a.cmd == "diff":
        print(json.dumps(diff(_load(a.before), _load(a.after)), indent=1))
    elif a.cmd == "show":
        inv = _load(a.inventory)
        for key, e in inv["kernels"].items():
            print(f"{e['work_share']:8.4f} {e['calls']:6d}  {key}" + (f"  FLAGS {e['flags']}" if e["flags"] else ""))
    return 0


if __name__ == "__main__":
    sys.exit(main())
