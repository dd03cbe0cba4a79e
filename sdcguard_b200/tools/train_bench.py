"""Training cost of the guard: GPT-2 small trained with and without `SDCGuard`, on one GPU.

    python -m sdcguard_b200.tools.train_bench --every 1 2 5 10 20 --steps 40 --warmup 5

Config (the reference's published GPT-2 small training measurement, results/round3_oct18/training/
fast_gpt2_overhead.json: 12 layers, 12 heads, d = 768, 512-token blocks, batch 32, AdamW at lr 6e-4): fp32
master weights, bf16 autocast, fused AdamW, synthetic token ids (random, uniform over the vocabulary), random-init
weights. The vocabulary is padded from 50257 to 50304 (a multiple of 128, common practice for GPT-2 training) so
the LM head, the largest GEMM, has a shape the checked GEMM takes; the reference's measurement reports 100 % of
matmuls checked.

Every arm trains its own copy of the same initial model for `warmup` untimed and `steps` timed steps. A step is
forward + loss + backward + optimizer step + zero_grad; its device time is taken with CUDA events around the
whole step and summed. With `--every N` every N-th step is checked: each nn.Linear's forward, dX and dW GEMMs run
on the checked tcgen05 GEMM with the ABFT check from its fp32 accumulator, the backward operands' checksum rows are
built on the device (`csrc/train_prep.cu`), and the guard reads the state table once per checked step. The line
reports the plain step time, each arm's mean step time and overhead, the cost of one checked step, and the checks,
alarms and worst clean score of the checked steps.

Reference: `SDCGuard` fast mode (src/sdcguard/guard.py:788, `protect` :1096); published overheads: +37.8 % every
step, +3.9 % every 10th step on an H100 (docs/METHOD.md:124-130).
"""
from __future__ import annotations

import argparse
import json
import time

import torch
import torch.nn.functional as F

from ..models.gpt2 import GPT2, GPT2Config


def _model(seed: int, vocab: int, dev) -> GPT2:
    torch.manual_seed(seed)
    return GPT2(GPT2Config(vocab=vocab), seed=seed).to(dev)


def _run(every: int, args, dev, batches) -> dict:
    from ..train.guard import SDCGuard
    model = _model(args.seed, args.vocab, dev)
    opt = torch.optim.AdamW(model.parameters(), lr=6e-4, weight_decay=0.1, betas=(0.9, 0.95), fused=True)
    guard = None
    if every > 0:
        guard = SDCGuard(check_every=every, device=dev)
        guard.protect(model)
    times, checked_times, losses = [], [], []
    total = args.warmup + args.steps
    for step in range(total):
        ids = batches[step % len(batches)]
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        ctx = guard.on_step(step) if guard is not None else _null()
        with ctx as checked:
            with torch.autocast("cuda", dtype=torch.bfloat16):
                logits = model(ids[:, :-1])
                loss = F.cross_entropy(logits.float().view(-1, logits.shape[-1]), ids[:, 1:].reshape(-1))
            loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=True)
        b.record()
        b.synchronize()
        if step >= args.warmup:
            t = a.elapsed_time(b)
            times.append(t)
            if checked:
                checked_times.append(t)
            losses.append(float(loss.detach()))
    out = {"every": every, "ms_per_step": sum(times) / len(times), "steps": len(times),
           "loss_first": losses[0], "loss_last": losses[-1]}
    if guard is not None:
        cov = guard.coverage()
        out.update(checked_steps=len(checked_times),
                   ms_per_checked_step=sum(checked_times) / max(1, len(checked_times)),
                   checks=cov["checks"], alarms=cov["alarms"], worst_clean_z=round(cov["worst_clean_z"], 4),
                   checked_calls=cov["checked_calls"], unchecked_calls=cov["unchecked_calls"],
                   alarm_examples=[{k: e.detail.get(k) for k in ("layer", "phase", "z", "row", "block")}
                                   for e in guard.events[:5]])
    del model, opt
    torch.cuda.empty_cache()
    return out


def profile_steps(args, dev, batches, every: int = 1) -> dict:
    """Kernel time of one plain and one checked step (torch.profiler CUDA activity; one launch list each): where a
    checked step's extra time goes."""
    from torch.profiler import ProfilerActivity, profile
    from ..train.guard import SDCGuard
    out = {}
    for name, checked in (("plain", False), ("checked", True)):
        model = _model(args.seed, args.vocab, dev)
        opt = torch.optim.AdamW(model.parameters(), lr=6e-4, fused=True)
        guard = SDCGuard(check_every=1, device=dev) if checked else None
        if guard is not None:
            guard.protect(model)

        def step(i):
            ctx = guard.on_step(i) if guard is not None else _null()
            with ctx:
                with torch.autocast("cuda", dtype=torch.bfloat16):
                    logits = model(batches[0][:, :-1])
                    loss = F.cross_entropy(logits.float().view(-1, logits.shape[-1]), batches[0][:, 1:].reshape(-1))
                loss.backward()
            opt.step()
            opt.zero_grad(set_to_none=True)
        for i in range(3):
            step(i)
        torch.cuda.synchronize()
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            t0 = time.perf_counter()
            step(3)
            torch.cuda.synchronize()
            wall = (time.perf_counter() - t0) * 1e3
        agg: dict = {}
        for e in prof.events():
            if e.device_type.name == "CUDA":
                k = e.name[:90]
                a = agg.setdefault(k, [0.0, 0])
                a[0] += e.device_time_total / 1e3 if hasattr(e, "device_time_total") else e.cuda_time_total / 1e3
                a[1] += 1
        top = sorted(agg.items(), key=lambda kv: -kv[1][0])[:15]
        out[name] = {"wall_ms": round(wall, 2), "kernel_ms": round(sum(v[0] for v in agg.values()), 2),
                     "launches": sum(v[1] for v in agg.values()),
                     "top": [[round(v[0], 3), v[1], k] for k, v in top]}
        del model, opt, guard
        torch.cuda.empty_cache()
    return out


class _null:
    def __enter__(self):
        return False

    def __exit__(self, *a):
        return False


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="sdcguard train-bench", description=__doc__.split("\n\n")[0])
    ap.add_argument("--every", type=int, nargs="+", default=[1, 10])
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--seq", type=int, default=512)
    ap.add_argument("--vocab", type=int, default=50304)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--profile", action="store_true", help="also profile one plain and one checked step")
    args = ap.parse_args(argv)
    dev = torch.device("cuda")
    torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = True
    g = torch.Generator(device=dev).manual_seed(args.seed + 1)
    batches = [torch.randint(0, args.vocab, (args.batch, args.seq + 1), device=dev, generator=g) for _ in range(8)]
    t0 = time.time()
    base = _run(0, args, dev, batches)
    arms = []
    for n in args.every:
        r = _run(n, args, dev, batches)
        r["overhead_pct"] = round(100.0 * (r["ms_per_step"] / base["ms_per_step"] - 1.0), 2)
        r["checked_step_extra_ms"] = round(r["ms_per_checked_step"] - base["ms_per_step"], 2)
        arms.append(r)
    from ..utils.gpuinfo import Sampler
    with Sampler(torch.cuda.current_device(), period_ms=200) as clk:
        _run(0, argparse.Namespace(**{**vars(args), "steps": 10, "warmup": 2}), dev, batches)
    prof = profile_steps(args, dev, batches) if args.profile else None
    print(json.dumps({"tool": "train_bench", "profile": prof, "model": "GPT-2 small (124M, vocab padded to %d)" % args.vocab,
                      "batch": args.batch, "seq": args.seq, "dtype": "bf16 autocast, fp32 master weights",
                      "data": "synthetic token ids", "gpu": torch.cuda.get_device_name(dev),
                      "plain_ms_per_step": round(base["ms_per_step"], 2), "arms": arms,
                      "clocks_plain_rerun": clk.summary(), "seconds": round(time.time() - t0, 1)}), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
