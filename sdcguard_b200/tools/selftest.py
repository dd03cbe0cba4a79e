"""`sdcguard selftest`: runs every checked kernel of the library once on a small case on one GPU and compares it
with a plain PyTorch fp32 computation of the same op; the checks must run and stay below the alarm line on clean
data, and an injected fault must be reported. Exit 0 when every item passes.

Reference counterpart: the reference's install self-check and `sdcguard demo` (src/sdcguard/demo.py), which run
its checks on a toy model; here every item is one of this library's sm_100a kernels.
"""
from __future__ import annotations

import argparse
import json
import time

import torch

from .. import _native
from ..numerics import abft
from ..ops import attention, gemm, kv_transfer, layers


def _gemm(dev) -> dict:
    g = torch.Generator().manual_seed(1)
    x = torch.randn(384, 1024, generator=g).to(dev, torch.bfloat16)
    w = (torch.randn(768, 1024, generator=g) * 0.02).to(dev, torch.bfloat16)
    cw = gemm.CheckedWeight(w)
    st = gemm.StateTable(dev, 4)
    s0, s1 = st.add("clean", cw.nb), st.add("injected", cw.nb)
    y = gemm.checked_linear(x, cw, st.state, s0)
    gemm.checked_linear(x, cw, st.state, s1, inject=(100, 300, 1 << 28))
    rows = st.read()
    err = ((y.float() - x.float() @ w.float().t()).abs().max() / (x.float() @ w.float().t()).abs().max()).item()
    ok = err < 1e-2 and rows[0]["z"] < abft.Z_ALARM and rows[0]["checks"] > 0 and rows[1]["z"] > abft.Z_ALARM \
        and rows[1].get("row") == 100 and rows[1].get("block") == 2
    return {"ok": ok, "max_rel_err": err, "clean_z": rows[0]["z"], "injected_z": rows[1]["z"]}


def _norm_act(dev) -> dict:
    g = torch.Generator().manual_seed(2)
    x = torch.randn(256, 1024, generator=g).to(dev, torch.bfloat16)
    w = (1 + 0.1 * torch.randn(1024, generator=g)).to(dev, torch.bfloat16)
    y, rs = layers.add_rmsnorm(x, w, 1e-6)
    xf = x.float()
    ref = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6)).bfloat16().float() * w.float()
    e1 = (y.float() - ref).abs().max().item()
    gu = torch.randn(256, 2 * 512, generator=g).to(dev, torch.bfloat16)
    a, _ = layers.silu_mul(gu)
    gf, uf = gu.float()[:, :512], gu.float()[:, 512:]
    e2 = (a.float() - torch.nn.functional.silu(gf) * uf).abs().max().item()
    rows = torch.arange(0, 256, 64, dtype=torch.int32, device=dev)
    st = torch.zeros(2, abft.STATE_COLS, dtype=torch.int64, device=dev)
    yr, _ = layers.add_rmsnorm(x, w, 1e-6, rows=rows)
    layers.compare_rows(y, rows, yr, st[0])
    bad = y.clone()
    bad.view(torch.int16)[64, 5] ^= 1
    layers.compare_rows(bad, rows, yr, st[1])
    z = [abft.decode_state_row(r)["z"] for r in st.cpu().tolist()]
    return {"ok": e1 < 0.05 and e2 < 0.05 and z[0] == 0 and z[1] > abft.Z_ALARM, "norm_err": e1, "act_err": e2,
            "replay_clean_z": z[0], "replay_flip_z": z[1]}


def _attention(dev) -> dict:
    g = torch.Generator().manual_seed(3)
    nq, nkv, n = 8, 2, 200
    pages = -(-n // 16)
    cache = torch.zeros(pages + 1, 2, nkv, 16, 128, dtype=torch.bfloat16, device=dev)
    kv = torch.randn(n, 2, nkv, 128, generator=g).to(dev, torch.bfloat16)
    for t in range(n):
        cache[1 + t // 16, :, :, t % 16] = kv[t]
    q = torch.randn(1, nq, 128, generator=g).to(dev, torch.bfloat16)
    bt = torch.arange(1, pages + 1, dtype=torch.int32, device=dev).view(1, -1)
    ctx = torch.tensor([n], dtype=torch.int32, device=dev)
    out = attention.decode(q, cache, bt, torch.zeros(1, dtype=torch.int32, device=dev), ctx, nq, nkv, 256)
    k, v = kv[:, 0].float(), kv[:, 1].float()
    grp = nq // nkv
    s = torch.einsum("hd,thd->ht", q[0].float(), k.repeat_interleave(grp, 1)) / 128 ** 0.5
    ref = torch.einsum("ht,thd->hd", s.softmax(-1), v.repeat_interleave(grp, 1))
    e = (out[0].float() - ref).abs().max().item()
    return {"ok": e < 0.02, "max_abs_err": e}


def _kv(dev) -> dict:
    cache = torch.randn(2, 9, 2, 2, 16, 128, device=dev).bfloat16()
    pages = torch.tensor([1, 4, 7], dtype=torch.int32, device=dev)
    sums = kv_transfer.page_checksums(cache, pages)
    got = [kv_transfer.as_u64(int(v)) for v in sums.cpu().tolist()]
    ref = [kv_transfer.page_checksum_reference(cache, int(p)) for p in pages.tolist()]
    return {"ok": got == ref}


ITEMS = {"gemm_abft": _gemm, "norm_act_replay": _norm_act, "decode_attention": _attention, "kv_page_checksum": _kv}


def run(device="cuda:0") -> dict:
    dev = torch.device(device)
    torch.cuda.set_device(dev)
    _native.lib()
    out = {}
    for name, fn in ITEMS.items():
        t0 = time.perf_counter()
        try:
            r = fn(dev)
        except Exception as e:          # an item that raises fails; the others still run
            r = {"ok": False, "error": f"{type(e).__name__}: {e}"}
        torch.cuda.synchronize(dev)
        r["seconds"] = round(time.perf_counter() - t0, 3)
        out[name] = r
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="sdcguard selftest")
    ap.add_argument("--device", default="cuda:0")
    ap.add_argument("--json", action="store_true")
    a = ap.parse_args(argv)
    if not torch.cuda.is_available():
        print("sdcguard selftest: no CUDA device")
        return 1
    res = run(a.device)
    if a.json:
        print(json.dumps(res, sort_keys=True, default=float))
    else:
        for k, r in res.items():
            print(f"{'PASS' if r['ok'] else 'FAIL'}  {k:18s} " + ", ".join(f"{kk}={vv}" for kk, vv in r.items()
                                                                              if kk != "ok"))
    return 0 if all(r["ok"] for r in res.values()) else 1
