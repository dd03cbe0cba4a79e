"""Microbenchmarks of single kernels (CUDA-event timing after warm-up, L2 flushed between timed launches), for
profiling and for the numbers in the profile summaries.

    python -m sdcguard_b200.tools.kernel_bench gemm --m 4096 --n 28672 --k 4096 [--iters 10]
    python -m sdcguard_b200.tools.kernel_bench gemm-timeline --m 256 --n 4096 --k 1024   # per-CTA phases
    python -m sdcguard_b200.tools.kernel_bench decode --batch 256 --nq 16 --nkv 8 --ctx 1600
    python -m sdcguard_b200.tools.kernel_bench prefill --seqs 8 --len 2048 --nq 16 --nkv 8

Each prints one JSON line: duration (median of the timed launches), achieved TFLOP/s or GB/s, and the cuBLAS
time of the same GEMM shape for reference.
"""
from __future__ import annotations

import argparse
import json
import os
import time

import torch

L2_FLUSH_BYTES = 256 << 20     # larger than the 126 MB L2


_CLOCKS: list = []        # clock summaries of the timed regions of this process (kept with the result)


def _timed(fn, iters: int, flush: bool = True, soak_s: float = 0.6) -> float:
    """Median CUDA-event time (ms) of `iters` launches after 3 warm-ups, L2 flushed before each; the SM clock is
    sampled (nvidia-smi, 100 ms) over the timed launches and a soak of the same launch of `soak_s` seconds, so
    every timing carries the clocks it ran at."""
    from ..utils.gpuinfo import Sampler
    buf = torch.empty(L2_FLUSH_BYTES, dtype=torch.int8, device="cuda") if flush else None
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    ts = []
    with Sampler(torch.cuda.current_device(), period_ms=100) as clk:
        for _ in range(iters):
            if buf is not None:
                buf.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            b.synchronize()
            ts.append(a.elapsed_time(b))
        t0 = time.time()
        while time.time() - t0 < soak_s:
            for _ in range(8):
                fn()
            torch.cuda.synchronize()
    _CLOCKS.append(clk.summary())
    ts.sort()
    return ts[len(ts) // 2]


def measured_peaks() -> dict:
    """The pool's measured roofline denominators (MEASURED_PEAKS.json at the repository root, written by the
    driver), or the earlier fallback measurement when it is absent."""
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                        "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured"}
    except (OSError, ValueError, KeyError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def bench_gemm(m, n, k, iters, bn=None):
    from ..ops import gemm
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(m, k, device=dev, generator=g).bfloat16()
    w = (torch.randn(n, k, device=dev, generator=g) * 0.02).bfloat16()
    cw = gemm.CheckedWeight(w)
    st = gemm.StateTable(dev, 2)
    s = st.add("gemm", cw.nb)
    rs = gemm.row_sqnorm(x)
    out = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
    ms = _timed(lambda: gemm.checked_linear(x, cw, st.state, s, row_sq=rs, out=out, bn=bn), iters)
    mc = _timed(lambda: torch.matmul(x, w.t(), out=out), iters)
    r = st.read()[0]
    fl = 2.0 * m * n * k
    return {"kernel": "checked_gemm", "m": m, "n": n, "k": k, "bn": bn or gemm.pick_bn(m, n, k=k), "us": round(ms * 1e3, 1),
            "tflops": round(fl / ms / 1e9, 1), "cublas_us": round(mc * 1e3, 1),
            "cublas_tflops": round(fl / mc / 1e9, 1), "worst_clean_z": round(r["z"], 4), "checks": r["checks"]}


DBG_SLOTS = 16     # per-CTA debug timer record of the checked GEMM (kDbgSlots in csrc/gemm_abft.cu)


def gemm_timeline(m, n, k, iters, bn=None):
    """Where a checked GEMM's time goes inside the kernel, from its per-CTA global-timer records (the kernel's
    debug timers: CTA start and end, time waiting for each accumulator, epilogue time, output-tile body, judge).
    Averages over CTAs of the median launch (L2 flushed before each); times in microseconds from the earliest
    CTA start. The timers cost a few loads and stores per tile; the launch is otherwise the production kernel, except
    that split-K is off while they run (shapes that would split over K show the unsplit kernel)."""
    from ..ops import gemm
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(m, k, device=dev, generator=g).bfloat16()
    w = (torch.randn(n, k, device=dev, generator=g) * 0.02).bfloat16()
    cw = gemm.CheckedWeight(w)
    st = gemm.StateTable(dev, 2)
    s = st.add("gemm", cw.nb)
    rs = gemm.row_sqnorm(x)
    out = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
    nsm = torch.cuda.get_device_properties(dev).multi_processor_count
    dbg = torch.zeros(nsm * DBG_SLOTS, dtype=torch.int64, device=dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.int8, device=dev)
    for _ in range(3):
        gemm.checked_linear(x, cw, st.state, s, row_sq=rs, out=out, bn=bn)
    runs = []
    for _ in range(max(1, iters)):
        flush.zero_()
        dbg.zero_()
        torch.cuda.synchronize()
        gemm.checked_linear(x, cw, st.state, s, row_sq=rs, out=out, bn=bn, dbg=dbg)
        torch.cuda.synchronize()
        d = dbg.view(nsm, DBG_SLOTS).cpu()
        d = d[d[:, 6] > 0]
        t0 = int(d[:, 5].min())
        runs.append({"ctas": int(d.shape[0]), "end_max_us": (int(d[:, 6].max()) - t0) / 1e3,
                     "end_mean_us": float((d[:, 6] - t0).double().mean()) / 1e3,
                     "tiles_per_cta": float(d[:, 2].double().mean()),
                     "wait_accumulator_us": float(d[:, 0].double().mean()) / 1e3,
                     "epilogue_us": float(d[:, 1].double().mean()) / 1e3,
                     "output_body_us": float(d[:, 3].double().mean()) / 1e3,
                     "judge_us": float(d[:, 4].double().mean()) / 1e3,
                     "body_tmem_load_wait_us": float(d[:, 7].double().mean()) / 1e3,
                     "body_staging_wait_us": float(d[:, 8].double().mean()) / 1e3,
                     "body_judge_prefetch_us": float(d[:, 9].double().mean()) / 1e3,
                     "body_sums_pack_us": float(d[:, 10].double().mean()) / 1e3,
                     "body_stage_store_us": float(d[:, 11].double().mean()) / 1e3})
    runs.sort(key=lambda r: r["end_max_us"])
    r = runs[len(runs) // 2]
    return {"kernel": "checked_gemm_timeline", "m": m, "n": n, "k": k,
            **{kk: round(v, 2) if isinstance(v, float) else v for kk, v in r.items()}}


def bench_fp8(m, n, k, iters):
    from ..ops import gemm
    from ..ops.fp8 import Fp8Weight, checked_linear_fp8, quantize_act
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(m, k, device=dev, generator=g).bfloat16()
    w = (torch.randn(n, k, device=dev, generator=g) * 0.02).bfloat16()
    fw = Fp8Weight(w)
    xa = quantize_act(x)
    st = gemm.StateTable(dev, 2)
    s = st.add("fp8", fw.nb)
    out = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
    ms = _timed(lambda: checked_linear_fp8(xa, fw, st.state, s, out=out), iters)
    mq = _timed(lambda: quantize_act(x, out=xa), iters)
    r = st.read()[0]
    fl = 2.0 * m * n * k
    res = {"kernel": "checked_gemm_fp8", "m": m, "n": n, "k": k, "us": round(ms * 1e3, 1),
           "tflops": round(fl / ms / 1e9, 1), "quant_us": round(mq * 1e3, 1), "worst_clean_z": round(r["z"], 4)}
    try:        # unchecked reference: torch's scaled fp8 matmul (per-tensor scales), when available
        a8 = x.float().clamp(-448, 448).to(torch.float8_e4m3fn)
        b8 = w.float().mul(64).clamp(-448, 448).to(torch.float8_e4m3fn)
        one = torch.ones((), device=dev)
        mt = _timed(lambda: torch._scaled_mm(a8, b8.t(), scale_a=one, scale_b=one, out_dtype=torch.bfloat16), iters)
        res.update(torch_scaled_mm_us=round(mt * 1e3, 1), torch_scaled_mm_tflops=round(fl / mt / 1e9, 1))
    except Exception as e:  # noqa: BLE001
        res["torch_scaled_mm"] = f"unavailable: {type(e).__name__}"
    return res


def bench_decode(batch, nq, nkv, ctx, iters):
    from ..ops import attention
    dev = torch.device("cuda")
    pages_per = -(-ctx // 16) + 1
    nblk = batch * pages_per + 1
    g = torch.Generator(device=dev).manual_seed(0)
    cache = torch.randn(nblk, 2, nkv, 16, 128, device=dev, generator=g).bfloat16()
    perm = torch.randperm(nblk - 1, device=dev, generator=g)[: batch * pages_per].int() + 1
    bt = perm.view(batch, pages_per).contiguous()
    q = torch.randn(batch, nq, 128, device=dev, generator=g).bfloat16()
    c = torch.full((batch,), ctx, dtype=torch.int32, device=dev)
    req = torch.arange(batch, dtype=torch.int32, device=dev)
    scratch = attention.decode_scratch(batch, nq, nkv, 4096, dev)
    out = torch.empty_like(q)
    ms = _timed(lambda: attention.decode(q, cache, bt, req, c, nq, nkv, 4096, out=out, scratch=scratch), iters)
    byts = batch * ctx * nkv * 2 * 256
    return {"kernel": "decode_attention", "batch": batch, "nq": nq, "nkv": nkv, "ctx": ctx, "us": round(ms * 1e3, 1),
            "gbs": round(byts / ms / 1e6, 1), "kv_bytes": byts}


def bench_prefill(seqs, length, nq, nkv, iters):
    from ..ops import attention
    dev = torch.device("cuda")
    pages_per = -(-length // 16)
    nblk = seqs * pages_per + 1
    g = torch.Generator(device=dev).manual_seed(0)
    cache = torch.randn(nblk, 2, nkv, 16, 128, device=dev, generator=g).bfloat16()
    bt = (torch.arange(seqs * pages_per, device=dev, dtype=torch.int32) + 1).view(seqs, pages_per)
    T = seqs * length
    q = torch.randn(T, nq, 128, device=dev, generator=g).bfloat16()
    pos = torch.arange(length, dtype=torch.int32, device=dev).repeat(seqs)
    tiles = attention.prefill_tiles([i * length for i in range(seqs)], [length] * seqs, nq // nkv).to(dev)
    out = torch.empty_like(q)
    ms = _timed(lambda: attention.prefill(q, cache, bt, pos, tiles, nq, nkv, out=out), iters)
    fl = 4.0 * seqs * nq * 128 * length * (length + 1) / 2       # causal QK^T and PV
    return {"kernel": "prefill_attention", "seqs": seqs, "len": length, "nq": nq, "nkv": nkv,
            "us": round(ms * 1e3, 1), "tflops": round(fl / ms / 1e9, 1)}


def bench_moe(tokens, experts, top_k, hidden, inter, iters):
    """Grouped checked gate_up GEMM of a MoE layer (every expert in one launch, rows grouped on the device) against
    PyTorch's grouped GEMM (`torch._grouped_mm`, unchecked) on the same grouped rows, plus the grouping kernels."""
    from ..ops import gemm, moe
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(tokens, hidden, device=dev, generator=g).bfloat16()
    ids = torch.stack([torch.randperm(experts, device=dev, generator=g)[:top_k] for _ in range(tokens)]).int()
    ws = [(torch.randn(2 * inter, hidden, device=dev, generator=g) * 0.02).bfloat16() for _ in range(experts)]
    stack = gemm.CheckedWeightStack(ws)
    grp = moe.Grouping(tokens, top_k, experts, hidden, dev)
    xg, rsq = grp.group(x, ids)
    st = gemm.StateTable(dev, 2)
    s = st.add("moe (ABFT GEMM)", stack.nb)
    out = torch.empty(grp.cap, 2 * inter, dtype=torch.bfloat16, device=dev)
    ms = _timed(lambda: gemm.checked_linear_grouped(xg, stack, grp.gband, grp.gcount, st.state, s, row_sq=rsq,
                                                    out=out), iters)
    mg = _timed(lambda: grp.group(x, ids), iters)
    rows = grp.expert_rows()
    pairs = tokens * top_k
    fl = 2.0 * pairs * hidden * 2 * inter
    r = {"kernel": "grouped_checked_gemm", "tokens": tokens, "experts": experts, "top_k": top_k, "hidden": hidden,
         "inter": inter, "padded_rows": int(grp.gcount.item()) * 128, "us": round(ms * 1e3, 1),
         "tflops": round(fl / ms / 1e9, 1), "grouping_us": round(mg * 1e3, 1),
         "weight_gbs": round(stack.weight.numel() * 2 / ms / 1e6, 1)}
    if hasattr(torch, "_grouped_mm"):
        # the same grouped rows, compact (no band padding), through PyTorch's grouped GEMM
        xc = torch.cat([xg[a:a + n] for a, n in rows])
        ends = torch.tensor([sum(n for _, n in rows[:e + 1]) for e in range(experts)], dtype=torch.int32,
                            device=dev)
        wt = torch.stack(ws).transpose(1, 2)
        try:
            mt = _timed(lambda: torch._grouped_mm(xc, wt, offs=ends), iters)
            r.update(torch_grouped_mm_us=round(mt * 1e3, 1), torch_grouped_mm_tflops=round(fl / mt / 1e9, 1))
        except (RuntimeError, TypeError, NotImplementedError) as e:
            r["torch_grouped_mm"] = f"unavailable: {type(e).__name__}: {str(e)[:120]}"
    row = st.read()[0]
    r.update(worst_clean_z=round(row["z"], 4), unjudged=row["unjudged"])
    return r


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m sdcguard_b200.tools.kernel_bench")
    sub = ap.add_subparsers(dest="what", required=True)
    a = sub.add_parser("gemm")
    a.add_argument("--m", type=int, default=4096)
    a.add_argument("--n", type=int, default=28672)
    a.add_argument("--k", type=int, default=4096)
    a.add_argument("--bn", type=int, default=None)
    t = sub.add_parser("gemm-timeline")
    t.add_argument("--m", type=int, default=256)
    t.add_argument("--n", type=int, default=4096)
    t.add_argument("--k", type=int, default=1024)
    t.add_argument("--bn", type=int, default=None)
    b = sub.add_parser("decode")
    b.add_argument("--batch", type=int, default=256)
    b.add_argument("--nq", type=int, default=16)
    b.add_argument("--nkv", type=int, default=8)
    b.add_argument("--ctx", type=int, default=1600)
    f = sub.add_parser("fp8")
    f.add_argument("--m", type=int, default=4096)
    f.add_argument("--n", type=int, default=28672)
    f.add_argument("--k", type=int, default=4096)
    c = sub.add_parser("prefill")
    c.add_argument("--seqs", type=int, default=8)
    c.add_argument("--len", type=int, default=2048)
    c.add_argument("--nq", type=int, default=16)
    c.add_argument("--nkv", type=int, default=8)
    mo = sub.add_parser("moe")
    mo.add_argument("--tokens", type=int, default=256)
    mo.add_argument("--experts", type=int, default=8)
    mo.add_argument("--top-k", type=int, default=2)
    mo.add_argument("--hidden", type=int, default=4096)
    mo.add_argument("--inter", type=int, default=14336)
    for p in (a, b, c, f, t, mo):
        p.add_argument("--iters", type=int, default=10)
    args = ap.parse_args(argv)
    if args.what == "gemm":
        r = bench_gemm(args.m, args.n, args.k, args.iters, args.bn)
    elif args.what == "gemm-timeline":
        r = gemm_timeline(args.m, args.n, args.k, args.iters, args.bn)
    elif args.what == "fp8":
        r = bench_fp8(args.m, args.n, args.k, args.iters)
    elif args.what == "decode":
        r = bench_decode(args.batch, args.nq, args.nkv, args.ctx, args.iters)
    elif args.what == "moe":
        r = bench_moe(args.tokens, args.experts, args.top_k, args.hidden, args.inter, args.iters)
    else:
        r = bench_prefill(args.seqs, args.len, args.nq, args.nkv, args.iters)
    peaks = measured_peaks()
    if _CLOCKS:
        r["clocks"] = _CLOCKS[0]
        if len(_CLOCKS) > 1:
            r["clocks_library"] = _CLOCKS[1]
    if "tflops" in r:
        r[f"fraction_of_{peaks['source']}_bf16"] = round(r["tflops"] / peaks["bf16_tflops"], 3)
    if "gbs" in r:
        r[f"fraction_of_{peaks['source']}_hbm"] = round(r["gbs"] / peaks["hbm_gbs"], 3)
    r["peaks"] = peaks
    print(json.dumps(r), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
