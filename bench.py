"""Headline benchmark: checked serving throughput on the Qwen3-0.6B-shaped decoder.

    python bench.py [--gpus N --steps K --warmup W] [--impl ours|reference]

One step = serving the whole load once: 256 requests, prompts uniform 1024-2048 tokens (synthetic ids), 128
generated tokens each, every GEMM ABFT-checked and a rotating 1/64 of rows of every other op replay-checked.
With N GPUs (one process per GPU, torchrun) every rank serves its own copy of the load (data-parallel replicas,
weak scaling); time is taken on the device with CUDA events, max over ranks; `value` is the job's total
tokens (prompt + generated) per second.

The JSON line also carries: the unchecked throughput of the same engine (cuBLAS GEMMs, no checks) and the
overhead; an end-to-end number through the public API (`LLMEngine.generate`, wall clock, pinned prompts in and
tokens out each step); a short fault-injection campaign (single-bit flips in GEMM accumulators, KV pages and
replayed rows) with the false alarms of the timed clean run; SM clocks sampled during the timed region.

--impl reference runs the unmodified reference package (baseline/_ref) through its public API on the same load:
`sdcguard.serve.ServeGuard().attach(model)` on a stock Hugging Face transformers Qwen3 model of the same shape
(random init, bf16), generating with `model.generate` in batches.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import torch

BASELINE_VALUE = None          # BASELINE.md has no published number for this config
METRIC = "checked tokens/s (prompt + generated) on Qwen3-0.6B-shaped serving, 256 req x 1024-2048 in / 128 out"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--requests", type=int, default=256)
    ap.add_argument("--new-tokens", type=int, default=128)
    ap.add_argument("--no-unchecked", action="store_true", help="skip the unchecked comparison run")
    ap.add_argument("--no-campaign", action="store_true", help="skip the fault-injection campaign")
    return ap.parse_args()


# ------------------------------------------------------------------------------------------ distributed
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                             device_id=torch.device("cuda", local))
    return rank, world, local


def barrier(world):
    if world > 1:
        torch.distributed.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t)
    return float(t.item())


# ------------------------------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi samples (200 ms) of this process's GPU during the timed region."""

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = f"/tmp/sdcguard_clocks_{os.getpid()}.csv"

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except Exception:  # noqa: BLE001
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:  # noqa: BLE001
                self.proc.kill()
            self.f.close()

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        try:
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx = float(parts[2])
                except ValueError:
                    continue
                for nm, v in zip(names, parts[5:9]):
                    if v.lower().startswith("active"):
                        reasons.add(nm)
        except OSError:
            pass
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------------------------------ workload
def make_load(n: int, seed: int = 1234, vocab: int = 151936):
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(1024, 2049, (n,), generator=g).tolist()
    prompts = torch.randint(0, vocab, (n, max(lens)), generator=g)
    return prompts, lens


def time_steps(fn, steps: int, world: int):
    """Device time (CUDA events, ms per step, max over ranks) and wall time of `steps` calls of fn."""
    barrier(world)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    a.record()
    for _ in range(steps):
        fn()
    b.record()
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    barrier(world)
    dev_ms = a.elapsed_time(b) / steps
    return max_over_ranks(dev_ms, world), max_over_ranks((t1 - t0) * 1000 / steps, world)


# ------------------------------------------------------------------------------------------ our arm
def run_ours(args, rank, world, local):
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from sdcguard_b200 import _native
    from sdcguard_b200.models.decoder import QWEN3_0_6B
    from sdcguard_b200.serve.engine import LLMEngine, PAGE
    cfg = QWEN3_0_6B
    prompts, lens = make_load(args.requests, seed=1234 + rank, vocab=cfg.vocab)
    prompts = prompts.pin_memory()
    tokens_per_step = sum(lens) + args.requests * args.new_tokens
    blocks = sum(-(-(n + args.new_tokens) // PAGE) for n in lens) + 64

    eng = LLMEngine(cfg, checked=True, num_blocks=blocks)
    out_box = {}

    def step():
        out_box["out"] = eng.generate(prompts, lens, args.new_tokens)

    for _ in range(args.warmup):
        step()
    eng.guard.poll()                                  # clear warm-up state; the timed run's alarms are counted
    _native.reset_launch_count()
    g0 = eng.graph_launches()
    with ClockSampler(local) as clk:
        dev_ms, wall_ms = time_steps(step, args.steps, world)
    launches = _native.launch_count() + eng.graph_launches() - g0
    events = eng.guard.poll()
    cov = eng.guard.coverage_report()
    false_alarms = int(sum_over_ranks(len(events), world))
    res = {"dev_ms": dev_ms, "wall_ms": wall_ms, "tokens_per_step": tokens_per_step, "clocks": clk.summary(),
           "launches": int(launches / max(1, args.steps)), "coverage": cov, "false_alarms": false_alarms}
    del eng
    torch.cuda.empty_cache()

    if not args.no_unchecked:
        ue = LLMEngine(cfg, checked=False, num_blocks=blocks)
        for _ in range(max(1, args.warmup)):
            ue.generate(prompts, lens, args.new_tokens)
        u_ms, _ = time_steps(lambda: ue.generate(prompts, lens, args.new_tokens), args.steps, world)
        res["unchecked_dev_ms"] = u_ms
        del ue
        torch.cuda.empty_cache()
    if not args.no_campaign:
        from sdcguard_b200.tools import campaign
        res["campaign"] = campaign.quick(seed=rank)
    return res


# ------------------------------------------------------------------------------------------ reference arm
def run_reference(args, rank, world, local):
    ref = os.path.join(os.path.dirname(os.path.abspath(__file__)), "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "sdcguard")):
        return {"unavailable": "reference not installed in baseline/_ref"}
    sys.path.insert(0, ref)
    from sdcguard.serve import ServeGuard      # the reference's public serving API
    from transformers import Qwen3Config, Qwen3ForCausalLM
    cfg = Qwen3Config(vocab_size=151936, hidden_size=1024, intermediate_size=3072, num_hidden_layers=28,
                      num_attention_heads=16, num_key_value_heads=8, head_dim=128, max_position_embeddings=40960,
                      rope_theta=1_000_000.0, rms_norm_eps=1e-6, tie_word_embeddings=True)
    torch.manual_seed(0)
    with torch.device("cuda"):
        model = Qwen3ForCausalLM(cfg).to(torch.bfloat16).eval()
    guard = ServeGuard().attach(model)
    prompts, lens = make_load(args.requests, seed=1234 + rank, vocab=cfg.vocab_size)
    prompts = prompts.pin_memory()
    tokens_per_step = sum(lens) + args.requests * args.new_tokens
    batch = int(os.environ.get("SDCGUARD_REF_BATCH", "64"))

    def step():
        outs = []
        for b0 in range(0, args.requests, batch):
            idx = list(range(b0, min(args.requests, b0 + batch)))
            L = max(lens[i] for i in idx)
            ids = torch.zeros(len(idx), L, dtype=torch.long)
            mask = torch.zeros(len(idx), L, dtype=torch.long)
            for j, i in enumerate(idx):           # left padding, as batched generation needs
                ids[j, L - lens[i]:] = prompts[i, :lens[i]]
                mask[j, L - lens[i]:] = 1
            ids = ids.pin_memory().to("cuda", non_blocking=True)
            mask = mask.pin_memory().to("cuda", non_blocking=True)
            with torch.no_grad():
                out = model.generate(input_ids=ids, attention_mask=mask, max_new_tokens=args.new_tokens,
                                     min_new_tokens=args.new_tokens, do_sample=False, pad_token_id=0)
            outs.append(out[:, L:].cpu())
        return outs

    for _ in range(args.warmup):
        step()
    guard.poll()
    with ClockSampler(local) as clk:
        dev_ms, wall_ms = time_steps(step, args.steps, world)
    events = guard.poll()
    return {"dev_ms": dev_ms, "wall_ms": wall_ms, "tokens_per_step": tokens_per_step, "clocks": clk.summary(),
            "false_alarms": int(sum_over_ranks(len(events), world))}


def main():
    args = parse()
    rank, world, local = dist_setup()
    n = world
    try:
        res = run_ours(args, rank, world, local) if args.impl == "ours" else run_reference(args, rank, world, local)
    finally:
        pass
    if rank == 0:
        base = {"n_gpus": n, "steps": args.steps, "warmup": args.warmup, "dtype": "bf16",
                "data": "synthetic (random token ids, random-init weights N(0,0.02))",
                "config": {"model": "Qwen3-0.6B-shaped (28 layers, d=1024, 16Q/8KV heads, head_dim 128, MLP 3072, "
                                    "vocab 151936)",
                           "global_batch": args.requests * n, "seq_len": "prompt U[1024,2048] + 128 generated",
                           "requests_per_gpu": args.requests, "kv_page_tokens": 16,
                           "parallelism": f"dp{n}" if n > 1 else "single GPU",
                           "l2": "inputs larger than L2 (KV cache ~48 GB per GPU, weights 1.2 GB)"}}
        if "unavailable" in res:
            line = {"impl": args.impl, "unavailable": res["unavailable"]}
        else:
            tps = n * res["tokens_per_step"] / (res["dev_ms"] / 1000.0)
            line = {"metric": METRIC, "value": round(tps, 1), "unit": "tokens/s", **base,
                    "ms_per_step": round(res["dev_ms"], 2), "higher_is_better": True, "scaling": "weak",
                    "vs_baseline": None if BASELINE_VALUE is None else round(tps / BASELINE_VALUE, 4),
                    "clocks": res["clocks"],
                    "e2e": {"value": round(n * res["tokens_per_step"] / (res["wall_ms"] / 1000.0), 1),
                            "unit": "tokens/s (wall clock through generate(), pinned prompts in, tokens out)",
                            "h2d_bytes_per_step": args.requests * 2048 * 8,
                            "d2h_bytes_per_step": args.requests * args.new_tokens * 8},
                    "false_alarms_clean_run": res["false_alarms"]}
            if args.impl == "reference":
                line["impl"] = "reference"
                line["checks"] = "reference ServeGuard on every nn.Linear (Triton check); no attention/KV checks"
            else:
                line["impl"] = "ours"
                line["gpu_launches"] = res["launches"]
                line["coverage"] = res["coverage"]
                if "unchecked_dev_ms" in res:
                    u = n * res["tokens_per_step"] / (res["unchecked_dev_ms"] / 1000.0)
                    line["unchecked_value"] = round(u, 1)
                    line["overhead_pct"] = round(100.0 * (u / tps - 1.0), 2)
                if "campaign" in res:
                    line["detection"] = res["campaign"]
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
