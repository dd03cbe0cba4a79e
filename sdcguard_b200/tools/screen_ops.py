"""Operator screen of one GPU: computations whose exact answer is known, compared bit for bit, plus matmuls of
realistic data judged against a stated bound and against a repeat of themselves.

    python -m sdcguard_b200.tools.screen_ops --minutes 2                  # cuda:0
    python -m sdcguard_b200.tools.screen_ops --minutes 1 --simulate fma_fp32   # what a failure report looks like

Tests (every value judged exactly unless stated):

  gemm_<p>        library matmuls in fp64, fp32 (TF32 off), tf32, bf16, fp16, fp8 (e4m3, `torch._scaled_mm`) and int8
                  (`torch._int_mm`) on integer-valued inputs in ranges where every product and partial sum is exact in
                  that arithmetic in any order, so the result is the exact integer (rounded once for bf16 / fp16
                  outputs). Each input set also runs scaled by exact powers of two and transposed.
  gemm_sdc_bf16,  this library's own tcgen05 kernels (checked bf16 GEMM, block-scaled fp8 GEMM) on the same kind of
  gemm_sdc_fp8    inputs: bf16 output equal to the exact result rounded once, and the kernel's own ABFT score clean.
  gemm_bf16_real, random-normal matmuls (every exponent and rounding the integer inputs never reach): sampled outputs
  gemm_fp16_real  against a float64 CPU reference within the output rounding plus 6 x the fp32 accumulation model,
                  and every output bit-identical to the same matmul run again.
  fma_fp32,       x * y + z on the CUDA cores with integer-valued operands generated in the kernel; the exact result
  fma_fp64        is formed on the integer units of the same thread (`csrc/screen.cu`).
  sm_consistency  special functions (exp, sin, tanh, rsqrt, log, an fp64 chain) of the same inputs computed twice by
                  different threads and SMs: the two results must be identical; a difference names both SMs.
  memory          a share of free memory filled with an address-dependent pattern and its complement, read back.

A single wrong value is a FAIL. The report gives test, round, input set, scaling, element, got and expected, and the
GPU's identity and telemetry before and after (nvidia-smi, read only). Exit code: 0 clean, 1 wrong values, 2 could
not run. `--simulate <test>` makes one value of that test's first round wrong on the host side (never a GPU fault).

Reference: src/sdcguard/screen_ops.py:1-57 (test families and exit codes), `run` :454.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import time
from typing import Optional

import torch

SMI_FIELDS = ("name", "uuid", "serial", "pci.bus_id", "driver_version", "vbios_version", "ecc.mode.current",
              "ecc.errors.corrected.volatile.total", "ecc.errors.uncorrected.volatile.total", "clocks.sm",
              "clocks.max.sm", "temperature.gpu", "power.draw", "clocks_event_reasons.active")
# value range r (inputs in [-r, r]) and inner size k per precision, with the bound that keeps every partial sum exact
EXACT = {
    "fp64": (2 ** 19, 1024),     # 2^38 * 2^10 = 2^48 < 2^53
    "fp32": (32, 2048),          # 2^10 * 2^11 = 2^21 < 2^24
    "tf32": (32, 2048),          # inputs below 2^11 are exact in TF32's 11-bit significand
    "bf16": (8, 2048),           # 2^6 * 2^11 = 2^17 < 2^24 (fp32 accumulation), output rounded once
    "fp16": (4, 2048),           # 2^4 * 2^11 = 2^15 < 65504
    "fp8": (3, 512),             # 9 * 2^9 < 2^13
    "int8": (127, 2048),         # 127^2 * 2^11 < 2^31
    "sdc_bf16": (8, 2048),
    "sdc_fp8": (3, 2048),        # scale 2^-7 per 128 block: 384 * 2^-7 = 3 exactly
}
SHAPES = ((1024, 1024, 1.0), (128, 4096, 1.0), (512, 1536, 0.5))     # (M, N, share of the precision's K)
POW2 = {"fp64": 300, "fp32": 40, "tf32": 40, "bf16": 40}            # +-exponent range of the exact scalings
REAL = ((16, 4096, 4096), (512, 1536, 2048), (256, 3072, 8960))
REAL_SAMPLES = 256
REAL_LINE = 2.0
FMA_N = 1 << 24
SM_N = 1 << 22
MAX_FIRST = 8


def smi(index: Optional[int]) -> dict:
    """nvidia-smi identity and telemetry of one GPU (read only; empty when unavailable)."""
    if index is None:
        return {}
    try:
        r = subprocess.run(["nvidia-smi", f"--id={index}", "--query-gpu=" + ",".join(SMI_FIELDS),
                            "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=20)
        lines = [x for x in r.stdout.splitlines() if x.strip()]
        return dict(zip(SMI_FIELDS, (v.strip() for v in lines[-1].split(",")))) if lines else {}
    except (OSError, subprocess.SubprocessError):
        return {}


class Found:
    """Wrong values of one test: count, checked values, and the first few with where to rerun them."""

    def __init__(self, name: str):
        self.name, self.wrong, self.checked, self.rounds, self.first, self.worst = name, 0, 0, 0, [], None

    def compare(self, got: torch.Tensor, want: torch.Tensor, where: dict) -> None:
        g, w = got.detach().reshape(-1), want.detach().reshape(-1).to(got.device)
        gb = g.view(_int_view(g.dtype)) if g.dtype.is_floating_point else g
        wb = w.to(g.dtype).view(_int_view(g.dtype)) if g.dtype.is_floating_point else w.to(g.dtype)
        bad = (gb != wb).nonzero().flatten()
        self.checked += g.numel()
        if bad.numel():
            self.wrong += int(bad.numel())
            for i in bad[: max(0, MAX_FIRST - len(self.first))].tolist():
                self.first.append({**where, "element": i, "got": _num(g[i]), "want": _num(w[i])})

    def add_record(self, rec: list, checked: int, where: dict) -> None:
        """A device-side record [wrong, index, got bits, want bits, sm a, sm b]."""
        self.checked += checked
        if rec[0]:
            self.wrong += rec[0]
            if len(self.first) < MAX_FIRST:
                self.first.append({**where, "element": rec[1], "got_bits": hex(rec[2] & (2 ** 64 - 1)),
                                   "want_bits": hex(rec[3] & (2 ** 64 - 1)), "sm": [rec[4], rec[5]]})

    def score(self, z: float) -> None:
        self.worst = z if self.worst is None else max(self.worst, z)

    def report(self) -> dict:
        d = {"wrong": self.wrong, "checked": self.checked, "rounds": self.rounds, "verdict":
             "FAIL" if self.wrong else "pass"}
        if self.worst is not None:
            d["worst_score"] = round(self.worst, 4)
        if self.first:
            d["first"] = self.first
        return d


def _int_view(dt: torch.dtype) -> torch.dtype:
    return {1: torch.uint8, 2: torch.int16, 4: torch.int32, 8: torch.int64}[dt.itemsize]


def _num(v: torch.Tensor):
    x = v.item()
    return x if isinstance(x, int) or math.isfinite(x) else str(x)


def _perturb(t: torch.Tensor, i: int = 3) -> torch.Tensor:
    """A copy with element i changed: its lowest significand bit flipped (floats) or +1 (integers)."""
    t = t.contiguous().clone()
    v = t.view(-1)
    if t.dtype.is_floating_point:
        v.view(_int_view(t.dtype))[i] ^= 1
    else:
        v[i] += 1
    return t


def _ints(gen: torch.Generator, shape, r: int) -> torch.Tensor:
    return torch.randint(-r, r + 1, shape, generator=gen, dtype=torch.int64)


def gemm_supported(p: str, device: torch.device) -> Optional[str]:
    if device.type != "cuda":
        return None if p in ("fp64", "fp32", "bf16") else "needs a GPU"
    if p == "fp8" and not hasattr(torch, "_scaled_mm"):
        return "torch._scaled_mm missing"
    if p == "int8" and not hasattr(torch, "_int_mm"):
        return "torch._int_mm missing"
    return None


class GemmSet:
    """One integer-valued input set of one precision, with its exact reference (computed once, float64 / int64)."""

    def __init__(self, p: str, m: int, n: int, k: int, seed: int, device: torch.device):
        self.p, self.mnk, self.device = p, (m, n, k), device
        r, _ = EXACT[p]
        g = torch.Generator().manual_seed(seed)
        a, b = _ints(g, (m, k), r), _ints(g, (k, n), r)
        self.want = a @ b                                          # exact in int64
        self.a, self.b = a, b

    def run(self, transposed: bool, e: int) -> tuple[torch.Tensor, torch.Tensor]:
        """(got, want) with the inputs scaled by 2^e (half on each side) and optionally transposed (B^T A^T)."""
        p, dev = self.p, self.device
        ea, eb = e // 2, e - e // 2
        if p == "int8":
            a, b = self.a.to(dev, torch.int8), self.b.to(dev, torch.int8)
            got = torch._int_mm(b.t().contiguous(), a.t().contiguous()).t() if transposed else torch._int_mm(a, b)
            return got, self.want.to(torch.int32)
        if p == "fp8":
            f8 = torch.float8_e4m3fn
            a, b = self.a.to(dev, torch.float32).to(f8), self.b.to(dev, torch.float32).to(f8)
            one = torch.ones((), device=dev)
            if transposed:     # (B^T A^T)^T: B^T row-major, A^T = a.t() is column-major already
                got = torch._scaled_mm(b.t().contiguous(), a.t(), scale_a=one, scale_b=one,
                                       out_dtype=torch.float32).t()
            else:
                got = torch._scaled_mm(a, b.t().contiguous().t(), scale_a=one, scale_b=one, out_dtype=torch.float32)
            return got, self.want.double()
        if p in ("sdc_bf16", "sdc_fp8"):
            return self._run_sdc(transposed)
        dt = {"fp64": torch.float64, "fp32": torch.float32, "tf32": torch.float32, "bf16": torch.bfloat16,
              "fp16": torch.float16}[p]
        a = (self.a.double() * 2.0 ** ea).to(dev, dt)
        b = (self.b.double() * 2.0 ** eb).to(dev, dt)
        prev = torch.backends.cuda.matmul.allow_tf32
        prev_r = torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction
        prev_h = torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction
        try:
            torch.backends.cuda.matmul.allow_tf32 = p == "tf32"
            torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = False
            torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = False
            got = (b.t() @ a.t()).t() if transposed else a @ b
        finally:
            torch.backends.cuda.matmul.allow_tf32 = prev
            torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = prev_r
            torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = prev_h
        return got, (self.want.double() * 2.0 ** e).to(dt)

    def _run_sdc(self, transposed: bool):
        """This library's kernels compute x @ W^T: x = A (m, k), W = B^T (n, k); transposed swaps the roles."""
        from ..ops import gemm
        dev = self.device
        x, w = (self.b.t(), self.a) if transposed else (self.a, self.b.t())
        want = self.want.t() if transposed else self.want
        st = gemm.StateTable(dev, 2)
        if self.p == "sdc_bf16":
            cw = gemm.CheckedWeight(w.to(dev, torch.bfloat16).contiguous())
            slot = st.add("screen", cw.nb)
            got = gemm.checked_linear(x.to(dev, torch.bfloat16).contiguous(), cw, st.state, slot)
        else:
            from ..ops.fp8 import Fp8Weight, checked_linear_fp8, quantize_act
            fw = Fp8Weight(w.to(dev, torch.bfloat16).contiguous())
            slot = st.add("screen", fw.nb)
            got = checked_linear_fp8(quantize_act(x.to(dev, torch.bfloat16).contiguous()), fw, st.state, slot)
        self.last_z = st.read()[0]["z"]
        return got, want.double().to(torch.bfloat16)


def real_round(dtype: torch.dtype, shape: tuple, seed: int, device, transposed: bool, found: Found,
               simulate: bool) -> None:
    """Random-normal matmul: REAL_SAMPLES outputs against float64, scored against the output rounding plus 6 x the
    fp32 accumulation model (a clean output scores at most 1); then the whole output against a repeat, bit for bit."""
    m, n, k = shape
    g = torch.Generator().manual_seed(seed)
    a, b = torch.randn(m, k, generator=g).to(dtype), torch.randn(k, n, generator=g).to(dtype)
    ad, bd = a.to(device), b.to(device)
    mm = (lambda: (bd.t() @ ad.t()).t()) if transposed else (lambda: ad @ bd)
    y1, y2 = mm(), mm()
    if simulate:
        y2 = _perturb(y2, 7)
    found.compare(y2, y1, {"shape": shape, "transposed": transposed, "what": "repeat"})
    idx = torch.randint(0, m * n, (REAL_SAMPLES,), generator=g)
    r, c = idx // n, idx % n
    ref = (a.double()[r] * b.double()[:, c].t()).sum(1)
    mag = (a.double()[r].abs() * b.double()[:, c].t().abs()).sum(1)
    u_out = 2.0 ** -8 if dtype == torch.bfloat16 else 2.0 ** -11
    bound = ref.abs() * u_out + 6 * 2.0 ** -24 * math.sqrt(k) * mag + 1e-30
    z = ((y1.double().cpu().view(-1)[idx] - ref).abs() / bound)
    found.score(float(z.max()))
    found.checked += REAL_SAMPLES
    bad = (z > REAL_LINE).nonzero().flatten()
    if bad.numel():
        found.wrong += int(bad.numel())
        for i in bad[:MAX_FIRST].tolist():
            found.first.append({"shape": shape, "transposed": transposed, "row": int(r[i]), "col": int(c[i]),
                                "score": float(z[i])})


def _lib():
    from .. import _native
    return _native


def fma_round(fp64: bool, n: int, seed: int, device, inject: int) -> list:
    nat = _lib()
    rec = torch.zeros(6, dtype=torch.int64, device=device)
    nat.check(nat.lib().sdc_screen_fma(n, seed, int(fp64), inject, rec.data_ptr(),
                                       torch.cuda.current_stream(device).cuda_stream), "screen fma")
    return rec.tolist()


def sm_round(n: int, seed: int, device, inject: int) -> list:
    nat = _lib()
    st = torch.cuda.current_stream(device).cuda_stream
    out = torch.empty(2, 2 * n, dtype=torch.int32, device=device)
    sm = torch.empty(2, n, dtype=torch.uint8, device=device)
    for p, shift in enumerate((0, n // 2 + 4099)):
        nat.check(nat.lib().sdc_screen_special(n, seed, shift, out[p].data_ptr(), sm[p].data_ptr(), st), "special")
    rec = torch.zeros(6, dtype=torch.int64, device=device)
    nat.check(nat.lib().sdc_screen_compare(n, out[0].data_ptr(), out[1].data_ptr(), sm[0].data_ptr(),
                                           sm[1].data_ptr(), inject, rec.data_ptr(), st), "compare")
    return rec.tolist()


def memory_test(device, share: float, seed: int, found: Found, limit_gb: float, inject: bool,
                chunk_mb: int = 512) -> None:
    """Fill `share` of free memory (at most limit_gb) chunk by chunk with the pattern, check every chunk; then the
    complement. Chunks stay allocated until both passes are done."""
    nat = _lib()
    st = torch.cuda.current_stream(device).cuda_stream
    free, _ = torch.cuda.mem_get_info(device)
    total = int(min(free * share, limit_gb * 2 ** 30)) // 8
    words = chunk_mb * 2 ** 20 // 8
    chunks, base = [], 0
    while base + words <= total:
        chunks.append((torch.empty(words, dtype=torch.int64, device=device), base))
        base += words
    for inv in (0, 1):
        for buf, b in chunks:
            nat.check(nat.lib().sdc_screen_mem_fill(buf.data_ptr(), words, b, seed, inv, st), "mem fill")
        for buf, b in chunks:
            rec = torch.zeros(6, dtype=torch.int64, device=device)
            inj = 12345 if (inject and inv == 0 and b == 0) else -1
            nat.check(nat.lib().sdc_screen_mem_check(buf.data_ptr(), words, b, seed, inv, inj, rec.data_ptr(), st),
                      "mem check")
            found.add_record(rec.tolist(), words, {"pass": "complement" if inv else "pattern", "chunk_base": b})
    found.rounds += 1
    del chunks


def _one_round(n: str, f: Found, sets: dict, rnd: int, seed: int, device, sim: bool, fma_n: int, sm_n: int,
               real) -> None:
    if n in sets:
        gs = sets[n][rnd % len(sets[n])]
        tr = bool(rnd // len(sets[n]) % 2)
        lo = POW2.get(gs.p, 0)
        e = 0 if lo == 0 else int(torch.randint(-lo, lo + 1, (1,),
                                                generator=torch.Generator().manual_seed(seed + rnd)))
        got, want = gs.run(tr, e)
        if sim:
            got = _perturb(got)
        f.compare(got, want, {"round": rnd, "set": rnd % len(sets[n]), "shape": gs.mnk,
                              "transposed": tr, "pow2": e})
        if hasattr(gs, "last_z"):
            f.score(gs.last_z)
    elif n.endswith("_real"):
        dt = torch.bfloat16 if "bf16" in n else torch.float16
        real_round(dt, real[rnd % len(real)], seed * 7 + rnd, device, bool(rnd // len(real) % 2), f, sim)
    elif n.startswith("fma_"):
        rec = fma_round(n == "fma_fp64", fma_n, seed * 131 + rnd, device, 5 if sim else -1)
        f.add_record(rec, fma_n, {"round": rnd})
    elif n == "sm_consistency":
        rec = sm_round(sm_n, seed * 17 + rnd, device, 9 if sim else -1)
        f.add_record(rec, sm_n, {"round": rnd})
    if n != "memory":
        f.rounds += 1


def run(device: torch.device, minutes: float = 1.0, seed: int = 0, tests=None, simulate: Optional[str] = None,
        mem_share: float = 0.25, mem_limit_gb: float = 16.0, fma_n: int = FMA_N, sm_n: int = SM_N,
        shapes=SHAPES, real=REAL) -> dict:
    t0 = time.time()
    cuda = device.type == "cuda"
    idx = device.index if cuda else None
    report = {"device": str(device), "torch": torch.__version__, "seed": seed, "minutes": minutes,
              "simulated": simulate, "telemetry_before": smi(idx) if cuda else {}, "tests": {}, "skipped": {}}
    if cuda:
        report["gpu"] = torch.cuda.get_device_name(device)
    names = [f"gemm_{p}" for p in ("fp64", "fp32", "tf32", "bf16", "fp16", "fp8", "int8", "sdc_bf16", "sdc_fp8")]
    names += ["gemm_bf16_real", "gemm_fp16_real", "fma_fp32", "fma_fp64", "sm_consistency", "memory"]
    names = [n for n in names if tests is None or n in tests]
    found = {}
    sets = {}
    for n in names:
        p = n[5:] if n.startswith("gemm_") else None
        why = None
        if p and not p.endswith("_real"):
            why = gemm_supported(p.replace("sdc_", "") if not p.startswith("sdc") else p, device)
            if p.startswith("sdc") and not cuda:
                why = "this library's kernels need a GPU"
        elif p and p.endswith("_real"):
            why = None if cuda or tests else "realistic-data matmuls are for GPUs (ask for them with --tests)"
        elif not cuda:
            why = "needs a GPU (native kernel)"
        if why:
            report["skipped"][n] = why
            continue
        found[n] = Found(n)
        if p and not p.endswith("_real"):
            r, kmax = EXACT[p]
            step = 128 if p.startswith("sdc") else 16
            sets[n] = [GemmSet(p, m, nn, max(step, int(kmax * ks) // step * step), seed * 1009 + 31 * i + len(n),
                               device)
                       for i, (m, nn, ks) in enumerate(shapes)]
    deadline = t0 + 60 * minutes
    rnd = 0
    try:
        if "memory" in found:
            memory_test(device, mem_share, seed, found["memory"], mem_limit_gb, simulate == "memory")
        while True:
            for n, f in list(found.items()):
                sim = simulate == n and rnd == 0
                try:
                    _one_round(n, f, sets, rnd, seed, device, sim, fma_n, sm_n, real)
                except RuntimeError as e:
                    if rnd:
                        raise
                    report["skipped"][n] = f"unsupported here: {str(e).splitlines()[0][:200]}"
                    del found[n]
            rnd += 1
            if time.time() >= deadline:
                break
        if "memory" in found:
            memory_test(device, mem_share, seed + 1, found["memory"], mem_limit_gb, False)
        if cuda:
            torch.cuda.synchronize(device)
    except Exception as e:  # noqa: BLE001  (reported; exit code 2)
        report["error"] = f"{type(e).__name__}: {e}"
    report["rounds"] = rnd
    report["tests"] = {n: f.report() for n, f in found.items()}
    report["telemetry_after"] = smi(idx) if cuda else {}
    report["seconds"] = round(time.time() - t0, 2)
    wrong = sum(f.wrong for f in found.values())
    report["verdict"] = "error" if "error" in report else ("FAIL" if wrong else "pass")
    return report


def exit_code(report: dict) -> int:
    return {"pass": 0, "FAIL": 1}.get(report["verdict"], 2)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m sdcguard_b200.tools.screen_ops", description=__doc__.split("\n")[0])
    ap.add_argument("--device", default="cuda:0" if torch.cuda.is_available() else "cpu")
    ap.add_argument("--minutes", type=float, default=1.0)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--tests", nargs="*")
    ap.add_argument("--simulate")
    ap.add_argument("--mem-share", type=float, default=0.25)
    ap.add_argument("--mem-limit-gb", type=float, default=16.0)
    ap.add_argument("--out", help="write the JSON report here")
    a = ap.parse_args(argv)
    rep = run(torch.device(a.device), a.minutes, a.seed, a.tests, a.simulate, a.mem_share, a.mem_limit_gb)
    text = json.dumps(rep, indent=1, default=str)
    if a.out:
        os.makedirs(os.path.dirname(os.path.abspath(a.out)), exist_ok=True)
        with open(a.out, "w") as f:
            f.write(text)
    print(json.dumps({"verdict": rep["verdict"], "tests": {k: v["verdict"] for k, v in rep["tests"].items()},
                      "skipped": rep["skipped"], "seconds": rep["seconds"]}))
    return exit_code(rep)


if __name__ == "__main__":
    raise SystemExit(main())
