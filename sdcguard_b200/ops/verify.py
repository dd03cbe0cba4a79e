"""First-use verification of this library's kernels on a device, before any result of theirs is trusted.

    report = verify.verified(torch.device("cuda:0"))     # cached per device; raises KernelNotVerified on failure

Each kernel family runs a small clean case and a corrupted one and is compared with a plain PyTorch restatement
in fp32 / fp64:

  gemm       the checked GEMM's output against an fp64 product (within bf16 rounding), no alarm on clean data, an
             injected accumulator exponent-bit flip reported at its (row, 128-column block)
  norm       add + RMSNorm against fp32, and its replay check finding one flipped output bit
  attention  paged prefill and decode against an fp32 softmax, and a prefill replay reproducing rows bit for bit
  spot       the spot check quiet on a clean output and reporting a flipped exponent bit where it is

A device whose kernels disagree is not used for checked serving or training (the engine refuses to start), which
is what the reference does before it trusts a Triton kernel on a GPU (src/sdcguard/_group.py:176 `verified`,
_serve_fast.py:639 and its probe :704, serve_attn.py:696 `verify_kernel`). The cases take well under a second.
"""
from __future__ import annotations

import math
import threading
import time

import torch

from ..numerics import abft

_lock = threading.Lock()
_DONE: dict = {}


class KernelNotVerified(RuntimeError):
    """A kernel of this library disagreed with its reference on this device."""


def _gemm_case(dev) -> dict:
    from . import gemm
    g = torch.Generator(device=dev).manual_seed(11)
    m, n, k = 192, 384, 512
    x = torch.randn(m, k, device=dev, generator=g).bfloat16()
    w = (torch.randn(n, k, device=dev, generator=g) * 0.05).bfloat16()
    b = (torch.randn(n, device=dev, generator=g) * 0.1).bfloat16()
    cw = gemm.CheckedWeight(w, b)
    table = gemm.StateTable(dev, 2)
    s0, s1 = table.add("clean (ABFT GEMM)", cw.nb), table.add("flip (ABFT GEMM)", cw.nb)
    y = gemm.checked_linear(x, cw, table.state, s0)
    gemm.checked_linear(x, cw, table.state, s1, inject=(37, 300, 1 << 29))
    torch.cuda.synchronize(dev)
    ref = x.double() @ w.double().t() + b.double()
    err = float(((y.double() - ref).abs() / (ref.abs() + 1e-2)).max())
    rows = table.read(reset=True)
    clean, flip = rows[s0], rows[s1]
    ok = err < 2 ** -7 and clean["z"] < abft.Z_ALARM and clean["unjudged"] == 0 and \
        flip["z"] > abft.Z_ALARM and flip.get("row") == 37 and flip.get("block") == 300 // 128
    return {"ok": bool(ok), "max_rel_err": err, "clean_z": clean["z"], "flip_z": flip["z"],
            "flip_at": (flip.get("row"), flip.get("block"))}


def _norm_case(dev) -> dict:
    from . import layers
    g = torch.Generator(device=dev).manual_seed(12)
    x = torch.randn(64, 1024, device=dev, generator=g).bfloat16()
    w = (1 + 0.1 * torch.randn(1024, device=dev, generator=g)).bfloat16()
    y, _ = layers.add_rmsnorm(x, w, 1e-6)
    xf = x.float()
    ref = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()
    err = float((y.float() - ref).abs().max())
    rows = torch.tensor([3, 40], dtype=torch.int32, device=dev)
    st = torch.zeros(2, abft.STATE_COLS, dtype=torch.int64, device=dev)
    layers.add_rmsnorm(x, w, 1e-6, out=y, rows=rows, check=st[0])
    bad = y.clone()
    bad.view(torch.int16)[40, 17] ^= 1
    layers.add_rmsnorm(x, w, 1e-6, out=bad, rows=rows, check=st[1])
    torch.cuda.synchronize(dev)
    clean, flip = abft.decode_state_row(st[0].tolist()), abft.decode_state_row(st[1].tolist())
    ok = err < 0.05 and clean["z"] == 0 and math.isinf(flip["z"])
    return {"ok": bool(ok), "max_abs_err": err, "replay_clean_z": clean["z"], "replay_flip_z": flip["z"]}


def _attention_case(dev) -> dict:
    from . import attention
    nq, nkv, blocks = 4, 2, 32
    g = torch.Generator(device=dev).manual_seed(13)
    cache = (torch.randn(blocks, 2, nkv, 16, 128, device=dev, generator=g) * 0.5).bfloat16()
    lens = [150, 70]
    bt = torch.zeros(2, 10, dtype=torch.int32, device=dev)
    bt[0, :10] = torch.arange(1, 11, dtype=torch.int32)
    bt[1, :5] = torch.arange(11, 16, dtype=torch.int32)
    T = sum(lens)
    q = (torch.randn(T, nq, 128, device=dev, generator=g) * 0.5).bfloat16()
    pos = torch.tensor(list(range(lens[0])) + list(range(lens[1])), dtype=torch.int32, device=dev)
    tiles = attention.prefill_tiles([0, lens[0]], lens, nq // nkv).to(dev)
    out = attention.prefill(q, cache, bt, pos, tiles, nq, nkv)
    # decode: one new token per sequence attending to its whole prefix
    qd = (torch.randn(2, nq, 128, device=dev, generator=g) * 0.5).bfloat16()
    ctx = torch.tensor(lens, dtype=torch.int32, device=dev)
    seq_req = torch.arange(2, dtype=torch.int32, device=dev)
    od = attention.decode(qd, cache, bt, seq_req, ctx, nq, nkv, 256)
    rt, ridx = attention.replay_tiles([[5, 149], [lens[0] + 60]], nq // nkv)
    rep = torch.zeros_like(out)
    attention.prefill(q, cache, bt, pos, rt.to(dev), nq, nkv, out=rep, row_idx=ridx.to(dev))
    torch.cuda.synchronize(dev)
    err, derr, starts = 0.0, 0.0, [0, lens[0]]
    for r, n in enumerate(lens):
        pages = bt[r, : -(-n // 16)].long()
        k = cache[pages, 0].permute(0, 2, 1, 3).reshape(-1, nkv, 128)[:n]
        v = cache[pages, 1].permute(0, 2, 1, 3).reshape(-1, nkv, 128)[:n]
        ref = attention.reference_attention(q[starts[r]:starts[r] + n], k, v, pos[starts[r]:starts[r] + n].long())
        err = max(err, float((out[starts[r]:starts[r] + n].float() - ref).abs().max()))
        refd = attention.reference_attention(qd[r:r + 1], k, v, torch.tensor([n - 1], device=dev))
        derr = max(derr, float((od[r:r + 1].float() - refd).abs().max()))
    exact = all(torch.equal(rep[t], out[t]) for t in ridx.tolist())
    ok = err < 0.02 and derr < 0.02 and exact
    return {"ok": bool(ok), "prefill_max_abs_err": err, "decode_max_abs_err": derr, "replay_bit_exact": exact}


def _spot_case(dev) -> dict:
    from . import gemm, spot
    g = torch.Generator(device=dev).manual_seed(14)
    x = torch.randn(64, 512, device=dev, generator=g).bfloat16()
    w = (torch.randn(256, 512, device=dev, generator=g) * 0.05).bfloat16()
    y = torch.matmul(x.float(), w.float().t()).bfloat16()
    rows = torch.arange(64, dtype=torch.int32, device=dev)
    cols = torch.tensor([1, 100, 255], dtype=torch.int32, device=dev)
    st = torch.zeros(2, abft.STATE_COLS, dtype=torch.int64, device=dev)
    spot.spot_check(x, w, y, rows, cols, st[0])
    bad = y.clone()
    bad.view(torch.int16)[9, 100] ^= 1 << 12
    spot.spot_check(x, w, bad, rows, cols, st[1])
    torch.cuda.synchronize(dev)
    clean, flip = abft.decode_state_row(st[0].tolist()), abft.decode_state_row(st[1].tolist())
    ok = clean["z"] == 0 and flip["z"] > abft.Z_ALARM and flip["flat"] == 9 * 256 + 100
    del gemm
    return {"ok": bool(ok), "clean_z": clean["z"], "flip_z": flip["z"], "flip_flat": flip["flat"]}


CASES = {"gemm": _gemm_case, "norm": _norm_case, "attention": _attention_case, "spot": _spot_case}


def run(device) -> dict:
    """Run every case now (no cache); {"ok", "device", "seconds", "cases": {name: {...}}}."""
    dev = torch.device(device)
    t0 = time.time()
    cases = {}
    with torch.cuda.device(dev):
        for name, fn in CASES.items():
            try:
                cases[name] = fn(dev)
            except Exception as e:  # noqa: BLE001  (a kernel that cannot run is not verified)
                cases[name] = {"ok": False, "error": f"{type(e).__name__}: {e}"}
    return {"ok": all(c["ok"] for c in cases.values()), "device": torch.cuda.get_device_name(dev),
            "index": dev.index if dev.index is not None else torch.cuda.current_device(),
            "seconds": round(time.time() - t0, 3), "cases": cases}


def verified(device, strict: bool = True) -> dict:
    """The cached verification report of `device` (run on first use). strict: raise KernelNotVerified when a
    kernel disagreed, naming the cases."""
    dev = torch.device(device)
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    with _lock:
        rep = _DONE.get(idx)
        if rep is None:
            rep = run(torch.device("cuda", idx))
            _DONE[idx] = rep
    if strict and not rep["ok"]:
        bad = {k: v for k, v in rep["cases"].items() if not v["ok"]}
        raise KernelNotVerified(f"sdcguard_b200 kernels disagree with their references on cuda:{idx}: {bad}")
    return rep
