"""`sdcguard check`: a short GPU health card. For a few minutes (or `--seconds`) it runs checked bf16 GEMMs through
the ABFT kernel and a device-to-device copy loop whose result is verified with the KV page checksum, and reports
throughput, the number of checks, the number of wrong results and the worst clean score.

Reference counterpart: `sdcguard check` (src/sdcguard/check.py:1530 `main`; the B200 card in the reference shows
bf16 8192^2 GEMM TFLOPS, D2D GB/s, results checked, wrong results and worst z). Board sharing, certificates and
provider detection are not part of this card.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import time

import torch

from .. import _native
from ..numerics import abft
from ..ops import gemm, kv_transfer


def _time(fn, iters: int) -> float:
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    fn()
    torch.cuda.synchronize()
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    b.synchronize()
    return a.elapsed_time(b) / iters


def run(device="cuda:0", seconds: float = 20.0, size: int = 8192, seed: int = 0) -> dict:
    dev = torch.device(device)
    torch.cuda.set_device(dev)
    _native.lib()
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(size, size, generator=g).to(dev, torch.bfloat16)
    w = (torch.randn(size, size, generator=g) * 0.02).to(dev, torch.bfloat16)
    cw = gemm.CheckedWeight(w)
    st = gemm.StateTable(dev, 2)
    slot = st.add("card", cw.nb)
    rs = gemm.row_sqnorm(x)
    y = torch.empty(size, size, dtype=torch.bfloat16, device=dev)
    flops = 2.0 * size ** 3
    ms_checked = _time(lambda: gemm.checked_linear(x, cw, st.state, slot, row_sq=rs, out=y), 10)
    ms_cublas = _time(lambda: torch.matmul(x, w.t()), 10)
    # copy loop: 2 GiB source, verified by page checksums on both sides
    pages = 4096
    src = torch.randint(-2 ** 15, 2 ** 15, (1, pages, 2, 8, 16, 128), dtype=torch.int16, device=dev).view(
        torch.bfloat16)
    dst = torch.empty_like(src)
    ms_copy = _time(lambda: dst.copy_(src), 10)
    idx = torch.arange(pages, dtype=torch.int32, device=dev)
    copies, wrong_copies = 0, 0
    t_end = time.time() + seconds
    gemms = 0
    while time.time() < t_end:
        for _ in range(20):
            gemm.checked_linear(x, cw, st.state, slot, row_sq=rs, out=y)
        gemms += 20
        dst.copy_(src)
        a = kv_transfer.page_checksums(src, idx)
        b = kv_transfer.page_checksums(dst, idx)
        wrong_copies += int((a != b).sum())
        copies += 1
    torch.cuda.synchronize()
    r = st.read()[0]
    # output fingerprint: the checked GEMM is deterministic, so every healthy GPU of a model gives the same bits
    gemm.checked_linear(x, cw, st.state, slot, row_sq=rs, out=y)
    fp = hashlib.sha256(y.view(torch.int16).cpu().numpy().tobytes()).hexdigest()[:32]
    from ..utils.events import device_identity
    ident = device_identity(dev)
    wrong = int(r["z"] > abft.Z_ALARM) + wrong_copies
    return {"device": torch.cuda.get_device_name(dev), "gemm_size": size, "seed": seed, "seconds": seconds,
            "result": "PASS" if wrong == 0 else "FAIL", "gpu_uuid": ident.get("gpu_uuid"),
            "pci_bus_id": ident.get("pci_bus_id"), "output_fingerprint": fp,
            "checked_gemm_tflops": round(flops / ms_checked / 1e9, 1), "cublas_gemm_tflops": round(flops / ms_cublas / 1e9, 1),
            "d2d_gbs": round(2 * src.numel() * 2 / ms_copy / 1e6, 1),
            "gemm_checks": r["checks"], "gemm_wrong": int(r["z"] > abft.Z_ALARM), "worst_z": round(r["z"], 3),
            "gemms": gemms, "copies_verified": copies * pages, "copies_wrong": wrong_copies}


SCHEMA = "sdcguard-b200-check/1"


def card(res: dict, device="cuda:0") -> dict:
    """A shareable card: the result, hashed hardware identity, versions, a fingerprint of the deterministic GEMM
    output keyed by the exact setup, and a digest of the card's contents (board.validate checks it)."""
    from .screen_ops import smi
    dev = torch.device(device)
    tel = smi(dev.index)
    ident = tel.get("uuid") or tel.get("serial") or ""
    c = {"schema": SCHEMA, "result": "PASS" if res["gemm_wrong"] == 0 and res["copies_wrong"] == 0 else "FAIL",
         "gpu": {"name": res["device"], "id_hash": hashlib.sha256(ident.encode()).hexdigest()[:16] if ident else None,
                 "driver": tel.get("driver_version")},
         "versions": {"torch": torch.__version__, "cuda": torch.version.cuda},
         "minutes": round(res["seconds"] / 60, 3),
         "speed": {"checked_tflops": res["checked_gemm_tflops"], "cublas_tflops": res["cublas_gemm_tflops"],
                   "d2d_gbs": res["d2d_gbs"]},
         "checked": {"gemm_checks": res["gemm_checks"], "copies_verified": res["copies_verified"],
                     "wrong": res["gemm_wrong"] + res["copies_wrong"], "worst_z": res["worst_z"]},
         "fingerprint": {"key": f"{res['device']}|{res['gemm_size']}|{res['seed']}|{torch.version.cuda}",
                         "output": res["output_fingerprint"]},
         "provider": os.environ.get("SDCGUARD_PROVIDER", "not stated")}
    c["digest"] = card_digest(c)
    return c


def card_digest(c: dict) -> str:
    body = {k: v for k, v in c.items() if k != "digest"}
    return hashlib.sha256(json.dumps(body, sort_keys=True, separators=(",", ":")).encode()).hexdigest()[:32]


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="sdcguard check")
    ap.add_argument("--device", default="cuda:0")
    ap.add_argument("--seconds", type=float, default=20.0)
    ap.add_argument("--size", type=int, default=8192)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--json", action="store_true")
    ap.add_argument("--share", help="write the shareable card (board input) to this file")
    a = ap.parse_args(argv)
    if not torch.cuda.is_available():
        print("sdcguard check: no CUDA device")
        return 1
    res = run(a.device, a.seconds, a.size, a.seed)
    if a.share:
        with open(a.share, "w") as f:
            json.dump(card(res, a.device), f, indent=1)
    if a.json:
        print(json.dumps(res, sort_keys=True))
    else:
        for k, v in res.items():
            print(f"{k:22s} {v}")
    return 0 if res["gemm_wrong"] == 0 and res["copies_wrong"] == 0 else 1
