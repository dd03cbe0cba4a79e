"""NVIDIA's listed cuBLAS wrong-result issues, matched against the cuBLAS this process loaded, the GPU and the mode.

    python -m sdcguard_b200.tools.known_issues           # this machine
    python -m sdcguard_b200.tools.known_issues --json

Verdicts per issue:
  applies       version, GPU and mode all match (for MPS issues: this process sees fewer SMs than the GPU has)
  may apply     version and GPU match; whether it bites depends on what the job runs (the issue's `when`)
  not active    version and GPU match, but the mode it needs is off here
  not affected  the version or the GPU is outside the issue's range

The table (`tools/data/cublas_issues.json`) restates NVIDIA's release notes; a version outside a listed range is not
proof of safety. This library's own checked paths do not use cuBLAS; the table matters for the unchecked arms and
for any library matmul a job still runs. Note issue 5807900 (library matmuls running concurrently with other kernels
that use Tensor Memory) on Blackwell: this library's tcgen05 kernels are such kernels.

Reference: src/sdcguard/known_issues.py:1-20 (verdicts, MPS detection), `affected` :184, `match` :273.
"""
from __future__ import annotations

import argparse
import ctypes
import fnmatch
import json
import os
from pathlib import Path
from typing import Optional

DATA = Path(__file__).resolve().parent / "data" / "cublas_issues.json"


def load() -> list[dict]:
    return json.loads(DATA.read_text())["issues"]


def _t(v) -> Optional[tuple]:
    return tuple(v) if v else None


def version_affected(issue: dict, ver: tuple) -> Optional[bool]:
    """True / False, or None when NVIDIA gives neither a first nor a fixed version."""
    intro, fixed = _t(issue.get("introduced")), _t(issue.get("fixed"))
    branch = issue.get("fixed_on_branch", {}).get(f"{ver[0]}.{ver[1]}")
    if branch is not None and ver >= tuple(branch):
        return False
    if intro is None and fixed is None:
        return None
    if intro is not None and ver < intro:
        return False
    if fixed is not None and ver >= fixed:
        return False
    return True


def cc_matches(issue: dict, cc: str) -> bool:
    pats = issue.get("cc")
    return pats is None or any(fnmatch.fnmatch(cc, p) for p in pats)


def cublas_version() -> Optional[tuple]:
    """cublasLtGetVersion() of the cuBLASLt this process has (torch's, once torch is imported)."""
    import torch  # noqa: F401  (loads torch's CUDA libraries first)
    for name in ("libcublasLt.so.12", "libcublasLt.so.13", "libcublasLt.so"):
        try:
            lib = ctypes.CDLL(name)
        except OSError:
            continue
        lib.cublasLtGetVersion.restype = ctypes.c_size_t
        v = int(lib.cublasLtGetVersion())
        return (v // 10000, v % 10000 // 100, v % 100)
    return None


def machine() -> dict:
    """cuBLAS version, compute capability, SM count seen vs the GPU's, and MPS settings of this process."""
    import torch
    out = {"cublas": cublas_version(), "cc": None, "sms_visible": None, "mps_percentage": None}
    if torch.cuda.is_available():
        p = torch.cuda.get_device_properties(0)
        out["cc"] = f"{p.major}.{p.minor}"
        out["sms_visible"] = p.multi_processor_count
        out["gpu"] = p.name
    pct = os.environ.get("CUDA_MPS_ACTIVE_THREAD_PERCENTAGE")
    out["mps_percentage"] = float(pct) if pct else None
    return out


def match(m: dict, issues: Optional[list] = None) -> list[dict]:
    issues = load() if issues is None else issues
    ver, cc = _t(m.get("cublas")), m.get("cc")
    res = []
    for it in issues:
        if ver is None or cc is None:
            verdict = "unknown"
        else:
            va = version_affected(it, ver)
            if not cc_matches(it, cc) or va is False:
                verdict = "not affected"
            elif it.get("needs") == "mps_partial":
                partial = m.get("mps_percentage") is not None and m["mps_percentage"] < 100
                verdict = "applies" if partial and va else ("not active" if va else "may apply")
            else:
                verdict = "may apply"
        res.append({"id": it["id"], "verdict": verdict, "summary": it["summary"], "when": it.get("when"),
                    "workaround": it.get("workaround")})
    return res


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m sdcguard_b200.tools.known_issues")
    ap.add_argument("--json", action="store_true")
    a = ap.parse_args(argv)
    m = machine()
    rows = match(m)
    if a.json:
        print(json.dumps({"machine": m, "issues": rows}))
    else:
        print(f"cuBLAS {m['cublas']}  compute capability {m['cc']}  MPS {m['mps_percentage']}")
        for r in rows:
            if r["verdict"] != "not affected":
                print(f"  {r['id']:10s} {r['verdict']:10s} {r['summary']}")
    return 1 if any(r["verdict"] == "applies" for r in rows) else 0


if __name__ == "__main__":
    raise SystemExit(main())
