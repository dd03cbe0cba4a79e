"""Upgrade gate for library GEMMs: keep a linear layer that computed wrong (or one known right) as a case, run the
cases on the stack installed now, and say what an upgrade of PyTorch, CUDA, cuBLAS or the driver changed.

    sdcguard gate capture --shape 1000,2048,16 --bias --pack gates/     a seeded linear layer run here, kept as a case
    sdcguard gate add evidence.pt --pack gates/                         a case from saved evidence
    sdcguard gate run gates/ --out before.json                          every case, each in a fresh process
    sdcguard gate compare before.json after.json                        a verdict per case
    sdcguard gate workaround gates/<case> --env KEY=VALUE ...           does setting these fix it here?
    sdcguard gate investigate gates/<case>                              does it follow a GPU or the software?
    sdcguard gate pin gates/<case> --out pin.csv                        a TunableOp file for the case's GEMM
    sdcguard gate model-ref / model-check                               the model gate (tools/gate_model.py)

(`sdcguard gate DIR --require checksum` is the KV-checksum coverage gate; the subcommands above are this tool.)

A run executes the recorded call (`torch.matmul` / `torch.addmm` of bf16, fp16 or fp32 operands, as F.linear
does) into an output filled with NaN, so elements the kernel never wrote are seen; each output is judged against a
float64 CPU reference with the bound u_out |ref| + k 2^-24 (|x| |w|^T) (+ the bias's rounding), which holds for
any fp32 accumulation order. Each case runs in a fresh process with cuBLASLt's Trace log on, so the kernel that ran
is read from the library (`tools/kernels.py` parses the log).

Verdicts (compare):
  PASSED        right in every run on both stacks
  REGRESSED     right in every run before, wrong at least once after
  UNCHANGED     wrong before and after, or right after only because another kernel ran (the failing one was
                avoided, not shown fixed)
  FIXED         wrong before, right after, the same kernel ran after, and the drop is significant (one-sided
                Fisher exact test, p < 0.01)
  INCONCLUSIVE  the conditions differ (GPU, SMs, GEMM-steering environment, PyTorch matmul flags: unknown never
                matches), fewer than 5 runs on a side, a run failed, a needed kernel log is missing, or no cases
Exit codes: 0 when every verdict is PASSED or FIXED (workaround: WORKS), 1 when one is REGRESSED or UNCHANGED
(DOESN'T WORK), 2 when one is INCONCLUSIVE or there was nothing to compare.

Reference: src/sdcguard/gate.py (the legacy upgrade gate; its case files, verdict words and exit codes are kept so
case packs and scripts carry over; the code here is this package's own).
"""
from __future__ import annotations

import argparse
import hashlib
import json
import math
import os
import subprocess
import sys
import tempfile
import time
from typing import Optional

CASE_SCHEMA = "sdcguard.gate/1"
RUN_SCHEMA = "sdcguard.gate-run/1"
MIN_RUNS = 5
FIXED_P = 0.01
UNIT = {"bfloat16": 2.0 ** -8, "float16": 2.0 ** -11, "float32": 2.0 ** -24}
STEER_PREFIXES = ("CUBLAS", "CUBLASLT_", "PYTORCH_TUNABLEOP_", "TORCH_CUBLASLT_", "CUDA_MPS_ACTIVE_THREAD")
STEER_NAMES = ("TORCH_BLAS_PREFER_CUBLASLT", "DISABLE_ADDMM_CUDA_LT", "NVIDIA_TF32_OVERRIDE",
               "CUDA_DEVICE_MAX_CONNECTIONS")
NOT_STEERING = ("CUBLASLT_LOG_LEVEL", "CUBLASLT_LOG_FILE", "CUBLASLT_LOG_MASK", "CUBLAS_LOGINFO_DBG",
                "CUBLAS_LOGDEST_DBG", "PYTORCH_TUNABLEOP_VERBOSE", "PYTORCH_TUNABLEOP_VERBOSE_FILENAME")
GOOD, BAD = ("PASSED", "FIXED"), ("REGRESSED", "UNCHANGED")


def steering_env(env=None) -> dict:
    """The environment variables that choose or change a GEMM kernel (log switches left out)."""
    env = os.environ if env is None else env
    return {k: env[k] for k in sorted(env)
            if (k.startswith(STEER_PREFIXES) or k in STEER_NAMES) and k not in NOT_STEERING}


def tunableop_path(name: str, gpu: int) -> str:
    """The file PyTorch's TunableOp uses for PYTORCH_TUNABLEOP_FILENAME=name on GPU `gpu`: the GPU number replaces
    a "%d", else goes before the last ".", else at the end (PyTorch's naming rule)."""
    d = str(int(gpu))
    if "%d" in name:
        return name.replace("%d", d, 1)
    dot = name.rfind(".")
    return name[:dot] + d + name[dot:] if dot >= 0 else name + d


def _sha_file(path: str) -> Optional[str]:
    try:
        with open(path, "rb") as f:
            return hashlib.sha256(f.read()).hexdigest()
    except OSError:
        return None


def inputs_digest(tensors: dict) -> str:
    """Content digest of a case's inputs: each name, dtype, shape and bytes (independent of the file layout)."""
    import torch
    h = hashlib.sha256()
    for name in sorted(tensors):
        t = tensors[name]
        h.update(name.encode() + b"\x00")
        if t is None:
            h.update(b"-\x00")
            continue
        c = t.detach().cpu().contiguous()
        h.update(f"{c.dtype}:{tuple(c.shape)}".encode() + b"\x00")
        if c.numel():
            h.update(c.view(-1).view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


# ------------------------------------------------------------------------------------------- one run (worker side)
def bound_and_ref(x, w, b, dtype: str):
    """float64 reference of x @ w^T (+ b) and the per-element bound of a correct result in `dtype`."""
    x64, w64 = x.double(), w.double()
    acc = x64 @ w64.t()
    ref = acc + (0 if b is None else b.double())
    k = x.shape[1]
    bound = UNIT[dtype] * ref.abs() + k * 2.0 ** -24 * (x64.abs() @ w64.abs().t()) + 1e-30
    if b is not None:       # a bias added after a first rounding of the product rounds twice
        bound = bound + UNIT[dtype] * acc.abs() + 2.0 ** -23 * b.double().abs()
    return ref, bound


def judge(y, ref, bound) -> dict:
    import torch
    yd = y.double().cpu()
    unwritten = int(torch.isnan(yd).sum())
    err = (yd - ref).abs()
    ok = torch.isfinite(yd) & (err <= bound)
    ratio = (err / bound).nan_to_num(nan=math.inf, posinf=math.inf)
    return {"wrong": int((~ok).sum()), "unwritten": unwritten, "nonfinite": int((~torch.isfinite(yd)).sum()),
            "worst_error_over_bound": float(ratio.max()) if ratio.numel() else 0.0}


def conditions(dev) -> dict:
    import torch
    cond = {"device_type": dev.type, "env": steering_env(),
            "matmul": {"bf16_reduced_precision_reduction": torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction,
                       "fp16_reduced_precision_reduction": torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction,
                       "tf32": torch.backends.cuda.matmul.allow_tf32,
                       "preferred_blas": str(torch.backends.cuda.preferred_blas_library())}}
    if dev.type == "cuda":
        p = torch.cuda.get_device_properties(dev)
        cond.update(gpu_name=p.name, compute_capability=f"{p.major}.{p.minor}", sms_visible=p.multi_processor_count)
    else:
        cond.update(gpu_name="cpu", compute_capability="cpu", sms_visible=0)
    return cond


def run_in_process(case_dir: str, repeats: int, device: Optional[str] = None) -> dict:
    import torch
    with open(os.path.join(case_dir, "case.json")) as f:
        case = json.load(f)
    if case.get("schema") != CASE_SCHEMA:
        raise ValueError(f"{case_dir}: not a {CASE_SCHEMA} case")
    op = case["op"]
    if op.get("call") != "linear":
        raise ValueError(f"{case_dir}: call {op.get('call')!r} is not supported")
    t = torch.load(os.path.join(case_dir, "inputs.pt"), map_location="cpu", weights_only=True)
    dt = getattr(torch, op["dtype"])
    x, w, b = t["x"].to(dt), t["w"].to(dt), t.get("bias")
    b = None if b is None else b.to(dt)
    ref, bound = bound_and_ref(x, w, b, op["dtype"])
    dev = torch.device(device or ("cuda" if torch.cuda.is_available() else "cpu"))
    xd, wd = x.to(dev), w.to(dev)
    bd = None if b is None else b.to(dev)
    y = torch.empty(x.shape[0], w.shape[0], dtype=dt, device=dev)
    runs = []
    with torch.no_grad():
        for _ in range(repeats):
            y.fill_(float("nan"))
            if bd is None:
                torch.matmul(xd, wd.t(), out=y)
            else:
                torch.addmm(bd, xd, wd.t(), out=y)
            if dev.type == "cuda":
                torch.cuda.synchronize(dev)
            runs.append(judge(y, ref, bound))
    from .casefile import stack
    return {"case": case["id"], "runs": runs, "n": len(runs), "conditions": conditions(dev), "stack": stack(),
            "outputs": int(y.numel()), "op": op, "inputs_sha256": inputs_digest({"x": t["x"], "w": t["w"],
                                                                               "bias": t.get("bias")})}


# ------------------------------------------------------------------------------------------- runs (parent side)
def kernels_from_log(text: str) -> dict:
    from .kernels import kernel_key, parse_line
    calls, ks = 0, {}
    for line in text.splitlines():
        try:
            c = parse_line(line)
        except ValueError:
            continue
        if c is None:
            continue
        calls += 1
        key = kernel_key(c)
        ks[key] = ks.get(key, 0) + 1
    return {"calls": calls, "kernels": ks}


def run_case(case_dir: str, repeats: int = 20, env: Optional[dict] = None, device: Optional[str] = None,
             timeout: float = 600.0) -> dict:
    """One case in a fresh process (the libraries read their environment once) with cuBLASLt's Trace log on."""
    case_dir = os.path.abspath(case_dir)
    with tempfile.TemporaryDirectory(prefix="sdcguard_gate_") as tmp:
        out, log = os.path.join(tmp, "result.json"), os.path.join(tmp, "lt.log")
        e = dict(os.environ)
        e.update(env or {})
        e.update(CUBLASLT_LOG_LEVEL="5", CUBLASLT_LOG_FILE=log)
        cmd = [sys.executable, "-m", "sdcguard_b200.tools.upgrade_gate", "--worker", case_dir, out, str(repeats),
               device or ""]
        try:
            p = subprocess.run(cmd, env=e, capture_output=True, text=True, timeout=timeout)
        except subprocess.TimeoutExpired:
            return {"case": os.path.basename(case_dir), "error": f"timed out after {timeout:.0f} s"}
        try:
            with open(out) as f:
                res = json.load(f)
        except (OSError, ValueError):
            return {"case": os.path.basename(case_dir),
                    "error": f"exit {p.returncode} without a result: {(p.stdout + p.stderr)[-600:]}"}
        try:
            with open(log, errors="replace") as f:
                res["kernel_log"] = {"log": True, **kernels_from_log(f.read())}
        except OSError:
            res["kernel_log"] = {"log": False, "calls": 0, "kernels": {}}
        res["applied_env"] = steering_env(env or {})
        return res


def bad_runs(res: dict) -> int:
    return sum(1 for r in res.get("runs", []) if r.get("wrong", 0) > 0 or r.get("unwritten", 0) > 0)


# ------------------------------------------------------------------------------------------- cases
def case_id(op: dict, cond: dict) -> str:
    gpu = "".join(ch for ch in str(cond.get("gpu_name") or "gpu").replace("NVIDIA", "") if ch.isalnum())[:12].lower()
    return f"{gpu or 'gpu'}-linear-{op['dtype']}-{op['n']}x{op['k']}x{op['m']}{'-bias' if op['bias'] else ''}"


def write_case(pack: str, op: dict, tensors: dict, cond: dict, stack: dict, observed: dict, kind: str, source: dict,
               kernels: Optional[dict] = None, name: Optional[str] = None) -> str:
    """Write a case without replacing another: the same inputs under the same id keep the first record; other
    inputs under a taken id get the id plus the start of their digest."""
    import torch
    cid = name or case_id(op, cond)
    digest = inputs_digest(tensors)
    for attempt in (cid, f"{cid}-{digest[:10]}"):
        d = os.path.join(pack, attempt)
        path = os.path.join(d, "case.json")
        if not os.path.exists(path):
            break
        try:
            with open(path) as f:
                if json.load(f).get("inputs", {}).get("content_sha256") == digest:
                    return d
        except (OSError, ValueError):
            pass
    else:
        return d
    os.makedirs(d, exist_ok=True)
    torch.save({k: (None if v is None else v.detach().cpu().contiguous()) for k, v in tensors.items()},
               os.path.join(d, "inputs.pt"))
    case = {"schema": CASE_SCHEMA, "id": os.path.basename(d), "kind": kind,
            "created": time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime()), "source": source, "op": op,
            "inputs": {"file": "inputs.pt", "sha256": _sha_file(os.path.join(d, "inputs.pt")),
                       "content_sha256": digest},
            "conditions": cond, "stack": stack, "kernels": kernels or {}, "observed": observed,
            "expected": {"reference": "float64 on the CPU", "bound": "output rounding + k x 2^-24 x |x||w|",
                         "prefill": "nan"}}
    with open(os.path.join(d, "case.json"), "w") as f:
        json.dump(case, f, indent=1, default=str)
    return d


def capture(shape, dtype="bfloat16", bias=True, pack="gates", seed=0, repeats=20, name=None, device=None) -> dict:
    """A seeded linear layer (out features n, in features k, tokens m) run here and kept: an incident when a run
    was wrong, else a pin (a shape known right here, to catch a regression)."""
    import torch
    n, k, m = shape
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g)
    w = torch.randn(n, k, generator=g) / math.sqrt(k)
    b = torch.randn(n, generator=g) if bias else None
    op = {"call": "linear", "dtype": dtype, "m": m, "n": n, "k": k, "bias": bias}
    tensors = {"x": x, "w": w, "bias": b}
    with tempfile.TemporaryDirectory(prefix="sdcguard_gate_new_") as tmp:
        d = write_case(tmp, op, tensors, {}, {}, {}, "pending", {"kind": "capture", "seed": seed}, name="case")
        res = run_case(d, repeats, device=device)
    if "error" in res:
        raise RuntimeError(res["error"])
    bad = bad_runs(res)
    observed = {"runs": res["n"], "runs_wrong": bad, "wrong_per_run": [r["wrong"] for r in res["runs"]],
                "outputs": res["outputs"]}
    kind = "incident" if bad else "pin"
    d = write_case(pack, op, tensors, res["conditions"], res["stack"], observed, kind,
                   {"kind": "capture", "seed": seed}, res["kernel_log"]["kernels"], name)
    return {"case": d, "kind": kind, "runs_wrong": bad, "runs": res["n"], "kernels": res["kernel_log"]["kernels"]}


def add(evidence: str, pack: str = "gates", name: Optional[str] = None) -> dict:
    """A case from saved evidence: a matmul's operands (A, B, C, bias with C = A @ B + bias: the reference's
    evidence files) or this package's casefile capture (x_row, w_block, y_block: one row and one 128-column block,
    a slice of the layer's GEMM, which the library may run with another kernel; the case says so)."""
    from ..utils.events import load_evidence
    ev = load_evidence(evidence)
    if "x_row" in ev:
        x, w, bias, dtype = ev["x_row"].view(1, -1), ev["w_block"], None, "bfloat16"
        note = "one row and one 128-column block of the layer's GEMM"
    elif all(k in ev for k in ("A", "B", "C")):
        if ev["A"].dim() != 2 or ev["B"].dim() != 2 or ev.get("batch") is not None:
            raise ValueError("only 2-D matmul evidence can be a case")
        if float(ev.get("alpha", 1.0)) != 1.0 or float(ev.get("beta", 1.0)) not in (0.0, 1.0):
            raise ValueError("only alpha = 1 and beta 0 or 1 (a linear layer) can be a case")
        x, w, bias = ev["A"], ev["B"].t(), ev.get("bias")
        dtype, note = str(ev["C"].dtype).replace("torch.", ""), None
    else:
        raise ValueError(f"{evidence}: no matmul operands in this evidence file")
    op = {"call": "linear", "dtype": dtype, "m": int(x.shape[0]), "n": int(w.shape[0]), "k": int(x.shape[1]),
          "bias": bias is not None}
    d = write_case(pack, op, {"x": x, "w": w, "bias": bias}, {"device_type": "cuda"}, {}, {"from_evidence": True},
                   "incident", {"kind": "evidence", "file": os.path.abspath(evidence),
                                "sha256": _sha_file(evidence), "note": note}, None, name)
    return {"case": d}


def cases(pack: str) -> list:
    return [os.path.join(pack, n) for n in sorted(os.listdir(pack))
            if os.path.isfile(os.path.join(pack, n, "case.json"))]


def run_pack(pack: str, repeats: int = 20, env: Optional[dict] = None, device: Optional[str] = None) -> dict:
    return {"schema": RUN_SCHEMA, "pack": os.path.abspath(pack), "repeats": repeats,
            "when": time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime()),
            "cases": {os.path.basename(d): run_case(d, repeats, env, device) for d in cases(pack)}}


# ------------------------------------------------------------------------------------------- verdicts
def fisher_one_sided(bad_a: int, n_a: int, bad_b: int, n_b: int) -> float:
    """P(at least bad_a failures among the first n_a runs) when bad_a + bad_b failures fall at random among all
    n_a + n_b runs (hypergeometric upper tail): small when the first side failed more than chance explains."""
    total, failures = n_a + n_b, bad_a + bad_b
    denom = math.comb(total, n_a)
    p = sum(math.comb(failures, i) * math.comb(total - failures, n_a - i)
            for i in range(bad_a, min(failures, n_a) + 1))
    return p / denom if denom else 1.0


def condition_differences(a: dict, b: dict, ignore_env=()) -> Optional[list]:
    """The conditions two runs differ in ([] when none); None when either run lacks one (unknown never matches)."""
    keys = ("gpu_name", "compute_capability", "sms_visible", "device_type")
    if any(a.get(k) is None or b.get(k) is None for k in keys) or a.get("env") is None or b.get("env") is None:
        return None
    diff = [k for k in keys if a[k] != b[k]]
    ea = {k: v for k, v in a["env"].items() if k not in ignore_env}
    eb = {k: v for k, v in b["env"].items() if k not in ignore_env}
    diff += [f"env {k}" for k in sorted(set(ea) | set(eb)) if ea.get(k) != eb.get(k)]
    ma, mb = a.get("matmul") or {}, b.get("matmul") or {}
    diff += [f"matmul {k}" for k in sorted(set(ma) | set(mb)) if ma.get(k) != mb.get(k)]
    return diff


def verdict(before: Optional[dict], after: Optional[dict], ignore_env=()) -> dict:
    for side, r in (("before", before), ("after", after)):
        if r is None:
            return {"verdict": "INCONCLUSIVE", "why": f"no run {side}"}
        if "error" in r:
            return {"verdict": "INCONCLUSIVE", "why": f"the run {side} failed: {r['error']}"}
        if r.get("n", 0) < MIN_RUNS:
            return {"verdict": "INCONCLUSIVE", "why": f"{r.get('n', 0)} runs {side} (at least {MIN_RUNS} needed)"}
    diff = condition_differences(before["conditions"], after["conditions"], ignore_env)
    if diff is None:
        return {"verdict": "INCONCLUSIVE", "why": "a run did not record its conditions"}
    if diff:
        return {"verdict": "INCONCLUSIVE", "why": "conditions differ: " + ", ".join(diff)}
    nb, na = bad_runs(before), bad_runs(after)
    counts = {"wrong_runs_before": nb, "runs_before": before["n"], "wrong_runs_after": na, "runs_after": after["n"]}
    if nb == 0:
        return {"verdict": "PASSED" if na == 0 else "REGRESSED", **counts}
    if na > 0:
        return {"verdict": "UNCHANGED", "why": "still wrong", **counts}
    kb, ka = before.get("kernel_log") or {}, after.get("kernel_log") or {}
    if not kb.get("log") or not ka.get("log") or not kb.get("kernels") or not ka.get("kernels"):
        return {"verdict": "INCONCLUSIVE", "why": "no kernel log to show the failing kernel ran after", **counts}
    if not set(kb["kernels"]) <= set(ka["kernels"]):
        return {"verdict": "UNCHANGED", "why": "avoided: another kernel ran after, the failing one was not shown fixed",
                **counts}
    p = fisher_one_sided(nb, before["n"], na, after["n"])
    if p >= FIXED_P:
        return {"verdict": "INCONCLUSIVE", "why": f"the drop in failures is not significant (p = {p:.3g})",
                "p": p, **counts}
    return {"verdict": "FIXED", "p": p, **counts}


def compare(a: dict, b: dict) -> dict:
    names = sorted(set(a.get("cases", {})) | set(b.get("cases", {})))
    per = {n: verdict(a.get("cases", {}).get(n), b.get("cases", {}).get(n)) for n in names}
    return {"cases": per, "exit": exit_code([v["verdict"] for v in per.values()])}


def exit_code(verdicts: list) -> int:
    if not verdicts or any(v == "INCONCLUSIVE" for v in verdicts):
        return 2
    if any(v in BAD for v in verdicts):
        return 1
    return 0


def workaround(case_dir: str, env: dict, repeats: int = 20, device: Optional[str] = None) -> dict:
    """The case without and with `env` set, on this stack: WORKS when it is wrong without and right with (the same
    significance rule as FIXED, the changed variables excepted from the condition match)."""
    base = run_case(case_dir, repeats, None, device)
    with_env = run_case(case_dir, repeats, env, device)
    if "error" not in base and bad_runs(base) == 0:
        return {"verdict": "INCONCLUSIVE", "why": "the case was right without the workaround (not reproduced)",
                "exit": 2}
    v = verdict(base, with_env, ignore_env=tuple(env))
    if v["verdict"] == "UNCHANGED" and "avoided" in v.get("why", ""):
        word = "WORKS"          # a workaround that steers to another kernel is exactly what it is for
    else:
        word = {"FIXED": "WORKS", "UNCHANGED": "DOESN'T WORK"}.get(v["verdict"], "INCONCLUSIVE")
    return {"verdict": word, "detail": v, "env": env, "exit": {"WORKS": 0, "DOESN'T WORK": 1}.get(word, 2)}


def investigate(case_dir: str, repeats: int = 20) -> dict:
    """The case on every visible GPU: DEVICE when only some are wrong, SOFTWARE PATH when all are, NOT REPRODUCED
    when none is."""
    import torch
    n = torch.cuda.device_count()
    per = {}
    for i in range(n):
        r = run_case(case_dir, repeats, None, f"cuda:{i}")
        per[f"cuda:{i}"] = {"wrong_runs": bad_runs(r), "runs": r.get("n", 0), "error": r.get("error"),
                            "kernels": (r.get("kernel_log") or {}).get("kernels")}
    bad = [d for d, r in per.items() if r["wrong_runs"] > 0]
    ok = [d for d, r in per.items() if r["wrong_runs"] == 0 and not r["error"]]
    word = ("NOT REPRODUCED" if not bad else "SOFTWARE PATH" if not ok else "DEVICE")
    return {"verdict": word, "gpus": per, "wrong_on": bad}


def pin(case_dir: str, out: str, repeats: int = 20, device: Optional[str] = None) -> dict:
    """Tune the case's GEMM with PyTorch's TunableOp into `out`, then run the case reading that file with tuning
    off: WORKS when the pinned kernel is right in every run."""
    import torch
    gpu = torch.device(device).index if device else 0
    tune_env = {"PYTORCH_TUNABLEOP_ENABLED": "1", "PYTORCH_TUNABLEOP_TUNING": "1",
                "PYTORCH_TUNABLEOP_FILENAME": out}
    tuned = run_case(case_dir, 1, tune_env, device)
    path = tunableop_path(out, gpu or 0)
    use_env = {**tune_env, "PYTORCH_TUNABLEOP_TUNING": "0"}
    pinned = run_case(case_dir, repeats, use_env, device)
    ok = "error" not in pinned and pinned.get("n", 0) >= MIN_RUNS and bad_runs(pinned) == 0
    return {"verdict": "WORKS" if ok else ("DOESN'T WORK" if "error" not in pinned else "INCONCLUSIVE"),
            "file": path, "file_sha256": _sha_file(path), "tuning_error": tuned.get("error"),
            "pinned_wrong_runs": bad_runs(pinned), "runs": pinned.get("n", 0),
            "kernels": (pinned.get("kernel_log") or {}).get("kernels")}


# ------------------------------------------------------------------------------------------- command line
def _env_pairs(items) -> dict:
    out = {}
    for it in items or []:
        k, sep, v = it.partition("=")
        if not sep:
            raise SystemExit(f"--env wants KEY=VALUE, got {it!r}")
        out[k] = v
    return out


def main(argv=None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    if argv and argv[0] == "--worker":
        case_dir, out, repeats = argv[1], argv[2], int(argv[3])
        device = argv[4] if len(argv) > 4 and argv[4] else None
        try:
            res = run_in_process(case_dir, repeats, device)
        except Exception as e:  # noqa: BLE001  (reported to the parent as the run's error)
            res = {"error": f"{type(e).__name__}: {e}"}
        with open(out, "w") as f:
            json.dump(res, f, indent=1, default=str)
        return 0
    ap = argparse.ArgumentParser(prog="sdcguard gate", description=__doc__.split("\n\n")[0])
    sub = ap.add_subparsers(dest="cmd", required=True)
    c = sub.add_parser("capture")
    c.add_argument("--shape", required=True, help="n,k,m: out features, in features, tokens")
    c.add_argument("--dtype", default="bfloat16", choices=sorted(UNIT))
    c.add_argument("--bias", action="store_true")
    c.add_argument("--pack", default="gates")
    c.add_argument("--seed", type=int, default=0)
    c.add_argument("--repeats", type=int, default=20)
    c.add_argument("--name")
    a = sub.add_parser("add")
    a.add_argument("evidence")
    a.add_argument("--pack", default="gates")
    a.add_argument("--name")
    r = sub.add_parser("run")
    r.add_argument("pack")
    r.add_argument("--out", required=True)
    r.add_argument("--repeats", type=int, default=20)
    r.add_argument("--env", nargs="*")
    cp = sub.add_parser("compare")
    cp.add_argument("before")
    cp.add_argument("after")
    cp.add_argument("--json", action="store_true")
    w = sub.add_parser("workaround")
    w.add_argument("case")
    w.add_argument("--env", nargs="+", required=True)
    w.add_argument("--repeats", type=int, default=20)
    iv = sub.add_parser("investigate")
    iv.add_argument("case")
    iv.add_argument("--repeats", type=int, default=20)
    pn = sub.add_parser("pin")
    pn.add_argument("case")
    pn.add_argument("--out", required=True)
    pn.add_argument("--repeats", type=int, default=20)
    for p in (c, r, w, pn):
        p.add_argument("--device")
    mr = sub.add_parser("model-ref")
    mc = sub.add_parser("model-check")
    for p in (mr, mc):
        p.add_argument("rest", nargs=argparse.REMAINDER)
    args = ap.parse_args(argv)
    if args.cmd in ("model-ref", "model-check"):
        from . import gate_model
        return gate_model.main(["ref" if args.cmd == "model-ref" else "check", *args.rest])
    if args.cmd == "capture":
        shape = tuple(int(v) for v in args.shape.split(","))
        if len(shape) != 3:
            raise SystemExit("--shape wants n,k,m")
        res = capture(shape, args.dtype, args.bias, args.pack, args.seed, args.repeats, args.name, args.device)
        print(json.dumps(res))
        return 0
    if args.cmd == "add":
        print(json.dumps(add(args.evidence, args.pack, args.name)))
        return 0
    if args.cmd == "run":
        res = run_pack(args.pack, args.repeats, _env_pairs(args.env), args.device)
        with open(args.out, "w") as f:
            json.dump(res, f, indent=1, default=str)
        wrong = {n: bad_runs(v) for n, v in res["cases"].items()}
        print(json.dumps({"out": args.out, "cases": len(wrong), "wrong_runs": wrong}))
        return 0 if res["cases"] else 2
    if args.cmd == "compare":
        with open(args.before) as f:
            before = json.load(f)
        with open(args.after) as f:
            after = json.load(f)
        res = compare(before, after)
        if args.json:
            print(json.dumps(res, indent=1))
        else:
            for n, v in res["cases"].items():
                print(f"{v['verdict']:13s} {n}" + (f"  ({v['why']})" if v.get("why") else ""))
            if not res["cases"]:
                print("INCONCLUSIVE  no cases")
        return res["exit"]
    if args.cmd == "workaround":
        res = workaround(args.case, _env_pairs(args.env), args.repeats, args.device)
        print(json.dumps(res))
        return res["exit"]
    if args.cmd == "investigate":
        res = investigate(args.case, args.repeats)
        print(json.dumps(res))
        return {"DEVICE": 1, "SOFTWARE PATH": 1}.get(res["verdict"], 2)
    res = pin(args.case, args.out, args.repeats, args.device)
    print(json.dumps(res))
    return {"WORKS": 0, "DOESN'T WORK": 1}.get(res["verdict"], 2)


if __name__ == "__main__":
    raise SystemExit(main())
