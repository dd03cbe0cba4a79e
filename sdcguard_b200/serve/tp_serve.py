"""Tensor-parallel checked serving run (one process per GPU, launched by torchrun): the Llama-3-8B-shaped decoder
split over the ranks (`models.tp_decoder.TPDecoder`), served by the paged-KV engine. The checked arm uses this
library's ABFT GEMMs and the sealed reduce-scatter / all-gather over NVLink peer memory; the unchecked arm is the
same model on cuBLAS GEMMs with NCCL collectives.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m sdcguard_b200.serve.tp_serve --batch 64 --prompt 2048 \
        --new-tokens 256

Rank 0 prints one JSON line: tokens/s of both arms (prompt + generated tokens over the device time of generate(),
max over ranks), the overhead, the check counts, false alarms on the clean run, agreement of the generated tokens
across ranks and arms, and the result of one injected flip in a reduce-scatter transfer.

Reference: TP in the reference is vLLM's, with local-shard checks only (src/sdcguard/guard.py:343-419,
_compiled.py:111-155); the collectives themselves carry no check there.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import time

import torch
import torch.distributed as dist

from .. import _native
from ..models.decoder import CONFIGS, LLAMA3_8B, TINY
from ..models.tp_decoder import TPDecoder
from ..parallel.symm import LocalHeap, SymmetricHeap
from ..parallel.tp import TPComm
from .engine import PAGE, LLMEngine


def _max(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _timed(fn, steps: int, world: int) -> tuple[float, float]:
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    a.record()
    for _ in range(steps):
        fn()
    b.record()
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    if world > 1:
        dist.barrier()
    return _max(a.elapsed_time(b) / steps, world), _max((t1 - t0) * 1000 / steps, world)


# kernels of the collectives (and the GEMMs fused with them) whose device time the profiled pass reports
COLLECTIVE_KERNELS = ("rs_pull_kernel", "ag_pull_kernel", "reduce_local", "add_rmsnorm_shard", "seal_rows_kernel",
                      "signal_kernel", "gemm_abft_kernel", "nccl", "nvjet", "cutlass")


def kernel_times(eng, prompts, lens, world: int, dev) -> dict:
    """Mean device time per launch (us, max over ranks) of the collective and GEMM kernels in one profiled short
    generate() (prefill of the whole batch, 4 decode steps), from the CUDA activity records of torch.profiler.
    Shares for reading where a step's time goes; the step's throughput is timed separately without the
    profiler."""
    from torch.profiler import ProfilerActivity, profile
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        eng.generate(prompts, lens, 5)
        torch.cuda.synchronize()
    rows = {}
    for e in prof.key_averages():
        t = getattr(e, "device_time_total", 0.0) or 0.0
        if t > 0 and any(k in e.key for k in COLLECTIVE_KERNELS):
            name = e.key.split("(")[0].replace("void ", "")[:80]
            rows[name] = {"launches": e.count, "us_per_launch": t / e.count, "total_us": t}
    names = sorted(rows)
    if world > 1:           # every rank reports the same names in the same order (max over ranks)
        objs = [None] * world
        dist.all_gather_object(objs, names)
        names = sorted(set().union(*objs))
        vals = torch.tensor([[rows.get(n, {}).get("us_per_launch", 0.0), rows.get(n, {}).get("total_us", 0.0)]
                             for n in names], dtype=torch.float64, device=dev).view(-1, 2)
        if vals.numel():
            dist.all_reduce(vals, op=dist.ReduceOp.MAX)
        return {n: {"launches": rows.get(n, {}).get("launches"), "us_per_launch": round(float(v[0]), 2),
                    "total_us": round(float(v[1]), 1)} for n, v in zip(names, vals.cpu())}
    return {n: {"launches": rows[n]["launches"], "us_per_launch": round(rows[n]["us_per_launch"], 2),
                "total_us": round(rows[n]["total_us"], 1)} for n in names}


def run(args) -> dict:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1 and not dist.is_initialized():     # (bench.py calls run() inside its own process group)
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=args.pg_timeout))
    cfg = CONFIGS.get(args.model) or {"llama3-8b": LLAMA3_8B, "tiny": TINY}[args.model]
    g = torch.Generator().manual_seed(args.seed)
    prompts = torch.randint(0, cfg.vocab, (args.batch, args.prompt), generator=g).pin_memory()
    lens = [args.prompt] * args.batch
    tokens_per_step = args.batch * (args.prompt + args.new_tokens)
    pages = args.batch * -(-(args.prompt + args.new_tokens) // PAGE) + 64
    max_rows = -(-max(args.max_prefill_tokens, args.batch) // world) * world
    heap = SymmetricHeap(device=dev) if world > 1 else LocalHeap(dev)
    comm = TPComm(heap, max_rows, cfg.hidden)
    res: dict = {"world": world}
    outs = {}
    for arm in args.arms.split(","):
        checked = arm == "checked"
        model = TPDecoder(cfg, comm if checked else None, rank, world, dev, checked=checked,
                          collective="own" if checked else "nccl", max_rows=max_rows, seed=args.seed,
                          precision=args.precision if checked else "bf16")
        eng = LLMEngine(cfg, dev, model=model, num_blocks=pages, max_prefill_tokens=args.max_prefill_tokens,
                        max_num_seqs=args.batch, max_model_len=args.prompt + args.new_tokens)
        box = {}

        def step():
            box["out"] = eng.generate(prompts, lens, args.new_tokens)

        for _ in range(args.warmup):
            step()
        eng.guard.poll()
        _native.reset_launch_count()
        g0 = eng.graph_launches()
        dev_ms, wall_ms = _timed(step, args.steps, world)
        launches = (_native.launch_count() + eng.graph_launches() - g0) // max(1, args.steps)
        eng.phase_timing = True
        step()
        eng.phase_timing = False
        phases = {k: round(_max(v, world), 2) for k, v in eng.last_phase_ms.items()}
        if getattr(args, "profile_kernels", False):
            r_k = kernel_times(eng, prompts, lens, world, dev)
        ev = eng.guard.poll()
        cov = eng.guard.coverage_report()
        outs[arm] = box["out"]
        r = {"dev_ms": dev_ms, "wall_ms": wall_ms, "tokens_per_s": tokens_per_step / (dev_ms / 1e3),
             "e2e_tokens_per_s": tokens_per_step / (wall_ms / 1e3), "gpu_launches": launches,
             "phase_ms": phases}
        if getattr(args, "profile_kernels", False):
            r["kernels"] = r_k
        if checked:
            r.update(checks=cov["checks"], unjudged=cov["unjudged"], worst_clean_z=cov["worst_clean_z"],
                     false_alarms=int(_max(len(ev), world)))
            # one injected flip in a reduce-scatter transfer: rank world-1 corrupts a sealed partial of its first
            # reduce-scatter in a short generate(); the owning rank must report it
            if args.inject:
                if rank == world - 1:
                    comm.inject_next(0, 5, 3)
                eng.generate(prompts[:1, :64].clone().pin_memory(), [64], 2)
                ev = eng.guard.poll()
                hit = [e.detail for e in ev if e.detector == "collective"]
                found = torch.tensor([1.0 if hit else 0.0], device=dev)
                if world > 1:
                    dist.all_reduce(found)
                r["injected_transfer_flip_detected_on_ranks"] = int(found.item())
                r["injected_flip_event"] = hit[0] if hit else None
        res[arm] = r
        del eng, model
        torch.cuda.empty_cache()
    if "checked" in outs and "unchecked" in outs:
        res["same_tokens_checked_vs_unchecked"] = float((outs["checked"] == outs["unchecked"]).float().mean())
    if world > 1:
        o = outs[next(iter(outs))].to(dev)
        allo = [torch.empty_like(o) for _ in range(world)]
        dist.all_gather(allo, o)
        res["ranks_agree"] = all(torch.equal(allo[0], x) for x in allo)
    if "checked" in res and "unchecked" in res:
        res["overhead_pct"] = round(100 * (res["checked"]["dev_ms"] / res["unchecked"]["dev_ms"] - 1), 2)
    comm.close()
    res["config"] = {"model": cfg.name, "tp": world, "precision": args.precision, "batch": args.batch,
                     "prompt": args.prompt,
                     "new_tokens": args.new_tokens, "steps": args.steps, "warmup": args.warmup}
    return res


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m sdcguard_b200.serve.tp_serve")
    ap.add_argument("--model", default="llama3-8b")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--prompt", type=int, default=2048)
    ap.add_argument("--new-tokens", type=int, default=256)
    ap.add_argument("--steps", type=int, default=1)
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--max-prefill-tokens", type=int, default=16384)
    ap.add_argument("--arms", default="checked,unchecked")
    ap.add_argument("--inject", action="store_true")
    ap.add_argument("--precision", default="bf16", choices=["bf16", "fp8"],
                    help="checked arm's projections: bf16, or block-scaled fp8 (the unchecked arm stays bf16)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--pg-timeout", type=int, default=300)
    ap.add_argument("--profile-kernels", action="store_true",
                    help="also report per-kernel device time of the collectives from one profiled short generate()")
    a = ap.parse_args(argv)
    res = run(a)
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps(res, default=str), flush=True)
    if dist.is_initialized():
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
