"""Expert-parallel checked serving step (one process per GPU, launched by torchrun): a Mixtral-8x7B-shaped model
(32 layers, d=4096, 32 Q / 8 KV heads, 8 experts top-2, expert FFN 14336, vocab 32000, random init) with data-parallel
attention and expert-parallel MoE layers. A step prefills 8192 tokens over the job (8192 / world per rank).

Arms: "checked" (ABFT GEMMs, exact replay checks, router replay, sealed all-to-all over NVLink peer memory) and
"unchecked" (cuBLAS GEMMs, NCCL all_to_all_single). Rank 0 prints one JSON line with tokens/s of both arms (device
time, max over ranks), the check counts and false alarms, and a seeded injection campaign: single-bit flips in expert
GEMM accumulators, in dispatched and returned all-to-all rows, and in KV-cache pages (verified by page checksums).

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m sdcguard_b200.serve.moe_serve
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import random
import time

import torch
import torch.distributed as dist

from .. import _native
from ..models.decoder import CheckedDecoder, DecoderConfig
from ..models.moe import MoELayer
from ..ops import kv_transfer
from ..parallel.ep import EPComm
from ..parallel.symm import LocalHeap, SymmetricHeap
from ..utils.inject import flip_bit_
from .engine import PAGE, LLMEngine

MIXTRAL = DecoderConfig("Mixtral-8x7B", 32, 4096, 32, 8, 128, 14336, 32000, 1_000_000.0, 1e-5, False,
                        max_position=32768)


def _max(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _sum(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t)
    return float(t.item())


def _timed(fn, steps, world):
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
    wall = (time.perf_counter() - t0) * 1000 / steps
    if world > 1:
        dist.barrier()
    return _max(a.elapsed_time(b) / steps, world), _max(wall, world)


def build(cfg, arm, comm, rank, world, dev, seed, precision: str = "bf16"):
    """precision "fp8" (checked arm): block-scaled fp8 expert GEMMs and attention projections; the unchecked
    baseline stays bf16 (PyTorch's grouped GEMM and cuBLAS)."""
    checked = arm == "checked"
    prec = precision if checked else "bf16"
    moe = [MoELayer(cfg.hidden, cfg.intermediate, 8, 2, comm if checked else None, dev, checked=checked,
                    seed=seed * 1000 + i, collective="own" if checked else "nccl", name=f"layers.{i}.moe",
                    precision=prec)
           for i in range(cfg.layers)]
    return CheckedDecoder(cfg, dev, checked=checked, seed=seed, moe_layers=moe, precision=prec), moe


def campaign(eng, model, moe, comm, rank, world, trials, seed, dev):
    """Seeded flips of each kind; a flip counts as detected when the check it targets reports it (on any rank)."""
    rng = random.Random(seed)
    T = 64
    g = torch.Generator().manual_seed(seed)
    prompts = torch.randint(0, model.cfg.vocab, (1, T), generator=g).pin_memory()
    res = {}

    def run_and_read():
        eng.generate(prompts, [T], 1)
        torch.cuda.synchronize()
        return eng.guard.poll()

    run_and_read()      # clean
    for kind in ("expert_gemm", "dispatch", "combine"):
        hits = 0
        for t in range(trials):
            layer = moe[rng.randrange(len(moe))]
            culprit = t % world
            if kind == "expert_gemm":
                if rank == culprit:
                    layer.inject_next("up", rng.randrange(4), rng.randrange(2 * model.cfg.intermediate),
                                      rng.choice([24, 27, 29, 30]))
            elif kind == "dispatch":
                if rank == culprit:
                    comm.inject_dispatch(rng.randrange(T * 2), rng.randrange(model.cfg.hidden), rng.randrange(7, 15))
            else:
                if rank == culprit:
                    comm.inject_combine(0, rng.randrange(model.cfg.hidden), rng.randrange(7, 15))
            ev = run_and_read()
            found = torch.tensor([1.0 if ev else 0.0], device=dev)
            if world > 1:
                dist.all_reduce(found, op=dist.ReduceOp.MAX)
            hits += int(found.item())
            # the injector fires on the next call whether or not this rank owned a token of the layer
        res[kind] = {"flips": trials, "detected": hits}
    # KV pages: checksums at prefill time, a flipped bit in a page, re-verification
    pages = eng.alloc.alloc(4)
    try:
        pg = torch.tensor(pages, dtype=torch.int32, device=dev)
        sums = kv_transfer.page_checksums(eng.cache, pg)
        hits = 0
        for t in range(trials):
            i = rng.randrange(len(pages))
            layer = rng.randrange(model.cfg.layers)
            page = eng.cache[layer, pages[i]]
            flat = rng.randrange(page.numel())
            flip_bit_(page, flat, rng.randrange(16))
            again = kv_transfer.page_checksums(eng.cache, pg)
            hits += int(bool((again != sums).any()))
            sums = again
        res["kv_page"] = {"flips": trials, "detected": hits}
    finally:
        eng.alloc.release(pages)
    return res


def run(args) -> dict:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1 and not dist.is_initialized():
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=args.pg_timeout))
    cfg = DecoderConfig(**{**MIXTRAL.__dict__, "layers": args.layers})
    T_local = args.tokens // world
    nseq = max(1, T_local // args.seq)
    lens = [T_local // nseq] * nseq
    g = torch.Generator().manual_seed(args.seed + rank)
    prompts = torch.randint(0, cfg.vocab, (nseq, lens[0]), generator=g).pin_memory()
    pages = sum(-(-(n + args.new_tokens) // PAGE) for n in lens) + 64
    heap = SymmetricHeap(device=dev) if world > 1 else LocalHeap(dev)
    comm = EPComm(heap, T_local, cfg.hidden, 8, 2)
    res: dict = {"world": world}
    for arm in args.arms.split(","):
        model, moe = build(cfg, arm, comm, rank, world, dev, args.seed, getattr(args, "precision", "bf16"))
        eng = LLMEngine(cfg, dev, model=model, num_blocks=pages, max_prefill_tokens=T_local, max_num_seqs=nseq,
                        cuda_graph=False, max_model_len=lens[0] + args.new_tokens)

        def step():
            eng.generate(prompts, lens, args.new_tokens)

        for _ in range(args.warmup):
            step()
        eng.guard.poll()
        _native.reset_launch_count()
        dev_ms, wall_ms = _timed(step, args.steps, world)
        launches = _native.launch_count() // max(1, args.steps)
        ev = eng.guard.poll()
        cov = eng.guard.coverage_report()
        tokens = args.tokens + world * nseq * (args.new_tokens - 1)
        r = {"dev_ms": round(dev_ms, 2), "tokens_per_s": round(tokens / (dev_ms / 1e3), 1),
             "e2e_tokens_per_s": round(tokens / (wall_ms / 1e3), 1), "gpu_launches": launches}
        if arm == "checked":
            r.update(checks=int(_sum(cov["checks"], world)), false_alarms=int(_sum(len(ev), world)),
                     worst_clean_z=round(_max(cov["worst_clean_z"], world), 4))
            if args.trials:
                r["injection"] = campaign(eng, model, moe, comm, rank, world, args.trials, args.seed, dev)
        res[arm] = r
        del eng, model, moe
        torch.cuda.empty_cache()
    if "checked" in res and "unchecked" in res:
        res["overhead_pct"] = round(100 * (res["checked"]["dev_ms"] / res["unchecked"]["dev_ms"] - 1), 2)
    comm.close()
    res["config"] = {"model": cfg.name, "layers": cfg.layers, "ep": world, "tokens_per_step": args.tokens,
                     "seq": lens[0], "new_tokens": args.new_tokens,
                     "dtype": ("fp8 block-scaled (checked arm), bf16 baseline" if getattr(args, "precision", "bf16") == "fp8"
                               else "bf16"), "steps": args.steps,
                     "warmup": args.warmup}
    return res


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m sdcguard_b200.serve.moe_serve")
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--tokens", type=int, default=8192)
    ap.add_argument("--seq", type=int, default=1024)
    ap.add_argument("--new-tokens", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--arms", default="checked,unchecked")
    ap.add_argument("--trials", type=int, default=8)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--pg-timeout", type=int, default=300)
    ap.add_argument("--precision", default="bf16", choices=["bf16", "fp8"],
                    help="fp8: block-scaled fp8 expert GEMMs and projections in the checked arm")
    a = ap.parse_args(argv)
    res = run(a)
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps(res, default=str), flush=True)
    if dist.is_initialized():
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
