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
At N = 1 it carries "train": the training guard's cost (GPT-2 small, every 10th step checked, against plain
training), measured in a process of its own. At N > 1 it carries three multi-GPU blocks, each timed on the device and taken as the max over ranks: "tp"
(the Llama-3-8B shape at TP = N, checked against cuBLAS + NCCL), and at even N "ep" (the Mixtral-8x7B shape at
EP = N, block-scaled fp8 checked against bf16 unchecked) and "pd" (prefill on N/2 ranks, decode on N/2, KV pages
pulled over NVLink with in-flight checksums, the coverage gate's verdict on each decode rank's recording). "ep" and
"pd" run as jobs of their own, one process per GPU, so a failure there leaves the headline standing.

--impl reference runs the unmodified reference package (installed in baseline/_ref) on its stock serving path, the
way its own vLLM experiments run it: vLLM's offline `LLM` engine on the same Qwen3-0.6B shape (random weights,
16-token KV blocks, prefix caching off so every step redoes every prompt), once with the reference's vLLM plugin
on (SDCGUARD=1: every linear layer checked by its Triton check, attention recompute on, stock settings) and once
with it off, each in a process of its own per GPU. The line reports the checked throughput as `value` and the
unchecked one beside it.
"""
from __future__ import annotations

import argparse
import gc
import json
import os
import signal
import socket
import statistics
import subprocess
import threading
import sys
import time

import torch

_T0 = time.monotonic()

BASELINE_VALUE = None          # no published number exists for this config
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
    ap.add_argument("--no-tp", action="store_true", help="skip the tensor-parallel block (config 4 at TP = N)")
    ap.add_argument("--no-tp-fp8", action="store_true", help="skip the block-scaled fp8 arm of the TP block")
    ap.add_argument("--tp-steps", type=int, default=1)
    ap.add_argument("--tp-batch", type=int, default=64)
    ap.add_argument("--tp-prompt", type=int, default=2048)
    ap.add_argument("--tp-new-tokens", type=int, default=256)
    ap.add_argument("--no-ep", action="store_true", help="skip the expert-parallel block (config 5 at EP = N)")
    ap.add_argument("--no-pd", action="store_true", help="skip the prefill/decode block (config 3 at N/2 + N/2)")
    ap.add_argument("--no-train", action="store_true", help="skip the training block (GPT-2 small, N = 1)")
    ap.add_argument("--ep-layers", type=int, default=4)
    ap.add_argument("--ep-steps", type=int, default=3)
    ap.add_argument("--block-limit", type=float, default=420.0,
                    help="seconds a multi-GPU block's processes may run before they are ended")
    ap.add_argument("--deadline", type=float, default=690.0,
                    help="seconds from start after which no multi-GPU block starts (each block's limit is cut to it)")
    ap.add_argument("--ref-child", choices=["checked", "unchecked"], help=argparse.SUPPRESS)
    ap.add_argument("--ref-rank", default="0", help=argparse.SUPPRESS)
    return ap.parse_args()


# ------------------------------------------------------------------------------------------ distributed
def dist_setup(use_gpu: bool = True):
    """Rank, world size and local rank from torchrun's environment; NCCL over this rank's GPU, or (for the
    reference arm, whose GPU belongs to the serving process it starts) gloo on the host."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if not use_gpu:
        if world > 1:
            import datetime
            torch.distributed.init_process_group("gloo", timeout=datetime.timedelta(seconds=1500))
        return rank, world, local
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
    if not args.no_tp and world > 1:
        try:
            res["tp"] = run_tp(args, world)
        except Exception as e:  # noqa: BLE001  (the headline line is printed with the TP block's error instead)
            res["tp"] = {"error": f"{type(e).__name__}: {str(e)[:300]}"}
    elif not args.no_tp:
        res["tp"] = {"skipped": "TP = 1 is the single-GPU engine of the headline; the block runs from N = 2"}
    gc.collect()
    torch.cuda.empty_cache()
    if world == 1 and not args.no_train:
        res["train"] = run_train(args)
    if world > 1 and world % 2 == 0:
        if not args.no_ep:
            res["ep"] = run_ep(args, rank, world, local)
        if not args.no_pd:
            res["pd"] = run_pd(args, rank, world, local)
    return res


# ------------------------------------------------------------------------------------------ multi-GPU blocks
def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def time_left(args) -> float:
    """Seconds left before the run's deadline, as rank 0 sees it (every rank takes the same decisions)."""
    cdev = "cuda" if torch.distributed.get_backend() == "nccl" else "cpu"
    t = torch.tensor([args.deadline - (time.monotonic() - _T0)], dtype=torch.float64, device=cdev)
    torch.distributed.broadcast(t, 0)
    return float(t.item())


def run_child_block(name: str, module: str, argv: list, rank: int, world: int, local: int, limit_s: float) -> dict:
    """Run one multi-GPU block as a job of its own: every rank starts one process of `module` on its GPU (a
    torch.distributed world of its own over a fresh loopback port, NVLS off), waits for it at most limit_s
    seconds, and the ranks agree on the outcome. A block that fails or hangs ends its processes and reports an
    error; the headline measured before it stands. Returns rank 0's JSON result (an empty dict elsewhere)."""
    cdev = "cuda" if torch.distributed.get_backend() == "nccl" else "cpu"     # (gloo in the CPU tests)
    port = torch.tensor([_free_port() if rank == 0 else 0], dtype=torch.int64, device=cdev)
    torch.distributed.broadcast(port, 0)
    env = {k: v for k, v in os.environ.items()
           if k not in ("GROUP_RANK", "ROLE_RANK", "ROLE_NAME", "ROLE_WORLD_SIZE", "GROUP_WORLD_SIZE")
           and not k.startswith(("TORCHELASTIC_", "TORCH_ELASTIC_"))}
    env.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(local), LOCAL_WORLD_SIZE=str(world),
               MASTER_ADDR="127.0.0.1", MASTER_PORT=str(int(port.item())), NCCL_NVLS_ENABLE="0",
               PYTHONPATH=os.path.dirname(os.path.abspath(__file__)) + os.pathsep + env.get("PYTHONPATH", ""))
    log_dir = os.environ.get("SDCGUARD_BLOCK_LOG_DIR", "/tmp")
    os.makedirs(log_dir, exist_ok=True)
    log_path = os.path.join(log_dir, f"sdcguard_block_{name}_{rank}.log")
    t0 = time.perf_counter()
    with open(log_path, "w") as log:
        p = subprocess.Popen([sys.executable, "-m", module, *argv], env=env, stdout=subprocess.PIPE, stderr=log,
                             text=True, start_new_session=True)
        try:
            out, _ = p.communicate(timeout=limit_s)
        except subprocess.TimeoutExpired:
            try:
                os.killpg(p.pid, signal.SIGKILL)
            except ProcessLookupError:          # it ended between the time-out and the kill
                pass
            out, _ = p.communicate()
    lines = [x for x in (out or "").splitlines() if x.startswith("{")]
    result = None
    if p.returncode == 0 and (rank != 0 or lines):
        try:
            result = json.loads(lines[-1]) if rank == 0 else {}
        except ValueError:
            result = None
    ok = torch.tensor([1 if result is not None else 0], dtype=torch.int64, device=cdev)
    torch.distributed.all_reduce(ok, op=torch.distributed.ReduceOp.MIN)
    if int(ok.item()) == 1:
        if rank == 0:
            result["block_wall_s"] = round(time.perf_counter() - t0, 1)
        return result
    if result is None:
        tail = open(log_path).read()[-600:].replace("\n", " | ")
        return {"error": f"{module} on rank {rank} ended with rc {p.returncode} after "
                         f"{time.perf_counter() - t0:.0f} s: {tail}"}
    return {"error": "another rank's process of this block failed (its log names the cause)"}


def run_train(args) -> dict:
    """The training guard's cost on one GPU, in a process of its own (its cuBLAS settings stay there): GPT-2 small
    (batch 32 x 512 tokens, AdamW, bf16 autocast) trained plainly and with every 10th step checked (each nn.Linear's
    forward, dX and dW GEMMs on the checked GEMM), device time per step with CUDA events."""
    left = args.deadline - (time.monotonic() - _T0)
    if left < 120:
        return {"skipped": f"{left:.0f} s left before the run's deadline"}
    cmd = [sys.executable, "-m", "sdcguard_b200.tools.train_bench", "--every", "10", "--steps", "40", "--warmup", "5"]
    env = dict(os.environ, PYTHONPATH=os.path.dirname(os.path.abspath(__file__)) + os.pathsep +
               os.environ.get("PYTHONPATH", ""))
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=min(args.block_limit, left))
    except subprocess.TimeoutExpired:
        return {"error": "the training block ran past its limit"}
    lines = [x for x in r.stdout.splitlines() if x.startswith("{")]
    if r.returncode != 0 or not lines:
        return {"error": f"rc {r.returncode}: " + r.stderr[-500:].replace("\n", " | ")}
    t = json.loads(lines[-1])
    arm = (t.get("arms") or [{}])[0]
    return {"model": t.get("model"), "batch": t.get("batch"), "seq": t.get("seq"), "dtype": t.get("dtype"),
            "plain_ms_per_step": t.get("plain_ms_per_step"), "checked_every": 10,
            "ms_per_step": arm.get("ms_per_step"), "overhead_pct": arm.get("overhead_pct"),
            "checked_step_extra_ms": arm.get("checked_step_extra_ms"),
            **{k: arm.get(k) for k in ("checks", "alarms", "worst_clean_z") if k in arm},
            "clocks": t.get("clocks_plain_rerun"), "seconds": t.get("seconds")}


def run_ep(args, rank: int, world: int, local: int) -> dict:
    """Config 5 on this job's GPUs: the Mixtral-8x7B-shaped model at EP = N (8 experts top-2 over N ranks,
    data-parallel attention, 8192 tokens per step over the job), the checked arm in block-scaled fp8 (grouped fp8
    checked expert GEMMs, sealed dispatch / combine all-to-all over NVLink peer memory, router and quantizer
    replays) against the bf16 unchecked arm (PyTorch grouped GEMM, NCCL all_to_all_single), device time max over
    ranks, plus seeded flips in expert GEMMs, dispatched and combined rows and KV pages."""
    argv = ["--layers", str(args.ep_layers), "--tokens", "8192", "--precision", "fp8", "--steps", str(args.ep_steps),
            "--warmup", "2", "--trials", "2", "--pg-timeout", "120"]
    left = time_left(args)
    if left < 150:
        return {"skipped": f"{left:.0f} s left before the run's deadline"}
    r = run_child_block("ep", "sdcguard_b200.serve.moe_serve", argv, rank, world, local, min(args.block_limit, left))
    if rank != 0 or "error" in r:
        return r
    c, u = r.get("checked", {}), r.get("unchecked", {})
    return {"config": r.get("config"), "ep": world, "unit": "tokens/s (whole job; device time max over ranks)",
            "checked_fp8": c.get("tokens_per_s"), "unchecked_bf16": u.get("tokens_per_s"),
            "overhead_pct": r.get("overhead_pct"),
            "ms_per_step": {"checked_fp8": c.get("dev_ms"), "unchecked_bf16": u.get("dev_ms")},
            "checks": c.get("checks"), "false_alarms": c.get("false_alarms"), "worst_clean_z": c.get("worst_clean_z"),
            "injection": c.get("injection"), "block_wall_s": r.get("block_wall_s")}


def run_pd(args, rank: int, world: int, local: int) -> dict:
    """Config 3 on this job's GPUs: prefill on the first N/2 ranks, decode on the other N/2 (4 + 4 at N = 8), 160
    requests in 8 shared-prefix groups on the Qwen3-0.6B shape, the decode ranks pulling KV pages from the producers'
    GPU memory with the checksumming copy. Two runs: clean (cached prefixes re-verified; the gate's verdict on every
    decode rank's recording) and with one bit flipped in a producer page (the pull must report it)."""
    out = {"prefill_ranks": world // 2, "decode_ranks": world // 2}
    # one directory for the job (the parent group's port names it), each decode rank writing its own decode<c>/
    rec_root = os.path.join(os.environ.get("SDCGUARD_BLOCK_LOG_DIR", "/tmp"),
                            f"sdcguard_pd_{os.environ.get('MASTER_PORT', '0')}_{world}")
    os.makedirs(rec_root, exist_ok=True)
    base = ["--prefill", str(world // 2), "--model", "Qwen3-0.6B", "--groups", "8", "--per-group", "20",
            "--new-tokens", "32", "--verify-cached-prefix", "--pg-timeout", "120"]
    for tag, extra in (("clean", ["--out", os.path.join(rec_root, "clean")]),
                       ("flipped_page", ["--out", os.path.join(rec_root, "flip"), "--corrupt-page", "0"])):
        left = time_left(args)
        if left < 100:
            out[tag] = {"skipped": f"{left:.0f} s left before the run's deadline"}
            continue
        r = run_child_block(f"pd_{tag}", "sdcguard_b200.serve.pd_mp", base + extra, rank, world, local,
                            min(args.block_limit, left))
        if rank != 0:
            continue
        if "error" in r:
            out[tag] = r
            continue
        out[tag] = {k: r.get(k) for k in ("requests", "tokens_per_s", "device_ms", "lifetime_violations",
                                          "ranks_with_mismatch", "kv_pull", "gate", "block_wall_s")}
    if rank == 0:
        clean, flip = out.get("clean", {}), out.get("flipped_page", {})
        gates = clean.get("gate") or []
        out["gate_pass_all_decode_ranks"] = bool(gates) and all(g.get("decision") == "PASS" for g in gates)
        out["flip_detected"] = ((flip.get("ranks_with_mismatch") or 0) >= 1
                                if flip and "error" not in flip and "skipped" not in flip else None)
    return out


def run_tp(args, world: int) -> dict:
    """Config 4 on this job's GPUs: the Llama-3-8B-shaped decoder at TP = N (batch 64, prompt 2048, 256 generated),
    checked (this library's GEMMs, the reduce-scatter pushed from the row-parallel GEMM's epilogue with seals, the
    sealed all-gather fused with the shard norm, all over NVLink peer memory) against unchecked (cuBLAS + NCCL),
    device time max over ranks, plus one profiled short generate() per arm for the collectives' device time."""
    import argparse as ap
    from sdcguard_b200.serve import tp_serve
    targs = ap.Namespace(model="llama3-8b", batch=args.tp_batch, prompt=args.tp_prompt,
                         new_tokens=args.tp_new_tokens, steps=args.tp_steps, warmup=1, max_prefill_tokens=16384,
                         arms="checked,unchecked", inject=True, precision="bf16", seed=0, pg_timeout=300,
                         profile_kernels=True)
    r = tp_serve.run(targs)
    c, u = r.get("checked", {}), r.get("unchecked", {})
    fp8 = None
    if not args.no_tp_fp8:
        # config 4 in block-scaled fp8: the checked arm again with the four projections on the fp8 checked GEMM
        # (1 x 128 activation and 128 x 128 weight scales), against the same bf16 unchecked arm
        try:
            f = tp_serve.run(ap.Namespace(**{**vars(targs), "arms": "checked", "precision": "fp8",
                                             "profile_kernels": False})).get("checked", {})
            fp8 = {"checked": round(f.get("tokens_per_s", 0.0), 1),
                   "overhead_pct_vs_bf16_unchecked": (round(100.0 * (u["tokens_per_s"] / f["tokens_per_s"] - 1.0), 2)
                                                      if f.get("tokens_per_s") and u.get("tokens_per_s") else None),
                   "ms_per_step": round(f.get("dev_ms", 0.0), 2), "checks": f.get("checks"),
                   "unjudged": f.get("unjudged"), "false_alarms": f.get("false_alarms"),
                   "injected_transfer_flip_detected_on_ranks": f.get("injected_transfer_flip_detected_on_ranks")}
        except Exception as e:  # noqa: BLE001  (the bf16 TP numbers stand; the fp8 arm reports its error)
            fp8 = {"error": f"{type(e).__name__}: {str(e)[:300]}"}
    return {"config": r.get("config"), "tp": world, "fp8": fp8,
            "checked": round(c.get("tokens_per_s", 0.0), 1),
            "unchecked": round(u.get("tokens_per_s", 0.0), 1), "overhead_pct": r.get("overhead_pct"),
            "unit": "tokens/s (prompt + generated, whole job; device time max over ranks)",
            "ms_per_step": {"checked": round(c.get("dev_ms", 0.0), 2), "unchecked": round(u.get("dev_ms", 0.0), 2)},
            "phase_ms": {"checked": c.get("phase_ms"), "unchecked": u.get("phase_ms")},
            "checks": c.get("checks"), "unjudged": c.get("unjudged"), "worst_clean_z": c.get("worst_clean_z"),
            "false_alarms": c.get("false_alarms"),
            "injected_transfer_flip_detected_on_ranks": c.get("injected_transfer_flip_detected_on_ranks"),
            "ranks_agree": r.get("ranks_agree"), "same_tokens_checked_vs_unchecked": r.get("same_tokens_checked_vs_unchecked"),
            "kernels_checked": c.get("kernels"), "kernels_unchecked": u.get("kernels"),
            "kernel_timing": "torch.profiler CUDA activity, one short generate (prefill + 4 decode steps) per arm"}


# ------------------------------------------------------------------------------------------ reference arm
QWEN3_0_6B_HF = {
    "architectures": ["Qwen3ForCausalLM"], "model_type": "qwen3", "hidden_size": 1024, "intermediate_size": 3072,
    "num_hidden_layers": 28, "num_attention_heads": 16, "num_key_value_heads": 8, "head_dim": 128,
    "vocab_size": 151936, "max_position_embeddings": 40960, "rope_theta": 1000000.0, "rms_norm_eps": 1e-06,
    "tie_word_embeddings": True, "torch_dtype": "bfloat16", "hidden_act": "silu", "attention_bias": False,
    "attention_dropout": 0.0, "bos_token_id": 151643, "eos_token_id": 151645, "use_cache": True,
    "use_sliding_window": False, "max_window_layers": 28, "initializer_range": 0.02,
}


def _ref_dir() -> str:
    return os.path.join(os.path.dirname(os.path.abspath(__file__)), "baseline", "_ref")


def _child_env(local: int, checked: bool) -> dict:
    """Environment of one reference serving process: this rank's GPU only, no torchrun variables (the engine
    builds its own one-process world), the reference package first on the path so vLLM finds its plugin entry
    point, and the plugin on (SDCGUARD=1, its stock defaults) or off."""
    # torchrun's variables, every TORCHELASTIC_* among them: with TORCHELASTIC_USE_AGENT_STORE set, torch's TCP
    # rendezvous connects as a client to a store the elastic agent would host, so the engine's own one-process
    # group would wait for a server that never starts
    env = {k: v for k, v in os.environ.items()
           if k not in ("RANK", "LOCAL_RANK", "WORLD_SIZE", "LOCAL_WORLD_SIZE", "GROUP_RANK", "ROLE_RANK",
                        "ROLE_NAME", "ROLE_WORLD_SIZE", "MASTER_ADDR", "MASTER_PORT", "GROUP_WORLD_SIZE")
           and not k.startswith(("TORCHELASTIC_", "TORCH_ELASTIC_"))}
    # this rank's GPU: the local-th entry of the job's visible devices (all ranks share the first one with
    # SDCGUARD_REF_SAME_GPU=1, which tests the multi-rank plumbing on one GPU)
    visible = [d for d in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if d.strip()]
    pick = 0 if os.environ.get("SDCGUARD_REF_SAME_GPU") == "1" else local
    env["CUDA_VISIBLE_DEVICES"] = visible[pick] if pick < len(visible) else str(pick)
    env["PYTHONPATH"] = _ref_dir() + os.pathsep + env.get("PYTHONPATH", "")
    env["VLLM_ENABLE_V1_MULTIPROCESSING"] = "0"       # engine core in this process: CUDA events see its work
    env["HF_HUB_OFFLINE"] = "1"
    env["TRANSFORMERS_OFFLINE"] = "1"
    env["VLLM_CACHE_ROOT"] = f"/tmp/sdcguard_ref_vllm_cache_{local}"
    env["VLLM_HOST_IP"] = "127.0.0.1"          # the engine's own one-process group over loopback
    env["SDCGUARD"] = "1" if checked else "0"
    return env


def ref_child(args) -> None:
    """One reference serving process (`bench.py --ref-child checked|unchecked`): vLLM's offline `LLM` on the
    Qwen3-0.6B shape (config only, random weights through vLLM's dummy loader, no tokenizer), prefix caching off
    so repeated steps redo every prompt, 16-token KV blocks. With SDCGUARD=1 vLLM loads the reference's plugin
    (its `vllm.general_plugins` entry point) and every linear layer and attention layer is checked as the
    reference ships it. Protocol on stdout/stdin: after the warm-up it prints READY and waits for a line GO, runs
    the timed steps, then prints its timings as one line `REFRESULT {json}`."""
    import torch
    from vllm import LLM, SamplingParams
    from vllm.inputs import TokensPrompt
    import vllm
    mdir = f"/tmp/sdcguard_ref_model_{os.getpid()}"
    os.makedirs(mdir, exist_ok=True)
    with open(os.path.join(mdir, "config.json"), "w") as f:
        json.dump(QWEN3_0_6B_HF, f)
    rank = int(args.ref_rank)
    prompts, lens = make_load(args.requests, seed=1234 + rank, vocab=QWEN3_0_6B_HF["vocab_size"])
    reqs = [TokensPrompt(prompt_token_ids=prompts[i, :lens[i]].tolist()) for i in range(args.requests)]
    sp = SamplingParams(max_tokens=args.new_tokens, min_tokens=args.new_tokens, ignore_eos=True, temperature=0.0)
    llm = LLM(model=mdir, load_format="dummy", skip_tokenizer_init=True, dtype="bfloat16", block_size=16,
              max_model_len=2048 + args.new_tokens, enable_prefix_caching=False, seed=0,
              gpu_memory_utilization=float(os.environ.get("SDCGUARD_REF_GPU_MEM", "0.85")))
    tokens_per_step = sum(lens) + args.requests * args.new_tokens
    h2d = sum(lens) * 8

    def step():
        outs = llm.generate(reqs, sp, use_tqdm=False)
        n = sum(len(o.outputs[0].token_ids) for o in outs)
        assert n == args.requests * args.new_tokens, f"generated {n} tokens"
        return outs

    for _ in range(args.warmup):
        step()
    plugin = None
    if os.environ.get("SDCGUARD") == "1":
        from sdcguard import vllm_plugin as plugin     # the reference's public read-back call
        plugin.poll(wait=True)
    print("READY", flush=True)
    sys.stdin.readline()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    a.record()
    for _ in range(args.steps):
        step()
    b.record()
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    alarms, checked_layers = 0, None
    if plugin is not None:
        alarms = len(plugin.poll(wait=True) or [])
        g = plugin.guard()
        checked_layers = len(getattr(g, "layers", []) or []) if g is not None else 0
    print("REFRESULT " + json.dumps({"dev_ms": a.elapsed_time(b) / args.steps, "wall_ms": (t1 - t0) * 1000 / args.steps,
                      "tokens_per_step": tokens_per_step, "h2d_bytes": h2d, "alarms": alarms,
                      "checked_layers": checked_layers, "vllm": vllm.__version__}), flush=True)


def _ref_phase(args, rank, world, local, checked: bool) -> dict:
    """Start this rank's reference serving process, wait for its READY, barrier over the ranks, release the timed
    steps together (GO), and collect its timings; clocks are sampled while it runs."""
    cmd = [sys.executable, os.path.abspath(__file__), "--ref-child", "checked" if checked else "unchecked",
           "--ref-rank", str(rank), "--steps", str(args.steps), "--warmup", str(args.warmup),
           "--requests", str(args.requests), "--new-tokens", str(args.new_tokens)]
    log_dir = os.environ.get("SDCGUARD_REF_LOG_DIR", "/tmp")
    os.makedirs(log_dir, exist_ok=True)
    log = open(os.path.join(log_dir, f"sdcguard_ref_{'c' if checked else 'u'}_{rank}.log"), "w")
    p = subprocess.Popen(cmd, env=_child_env(local, checked), stdin=subprocess.PIPE, stdout=subprocess.PIPE,
                         stderr=log, text=True)
    # the engine must report READY within SDCGUARD_REF_START_S seconds (default 600): a watchdog ends a child that
    # hangs in its startup, so every rank reaches the agreement below in bounded time and the line names the cause
    start_limit = float(os.environ.get("SDCGUARD_REF_START_S", "600"))
    ready_seen = threading.Event()

    def watchdog():
        if not ready_seen.wait(start_limit) and p.poll() is None:
            p.kill()
    threading.Thread(target=watchdog, daemon=True).start()
    ok = False
    for line in p.stdout:
        if line.strip() == "READY":
            ok = True
            ready_seen.set()
            break
    flag = torch.tensor([1 if ok else 0], dtype=torch.int64)
    if world > 1:
        torch.distributed.all_reduce(flag, op=torch.distributed.ReduceOp.MIN)
    res = None
    if int(flag.item()) == 1:
        with ClockSampler(local) as clk:
            p.stdin.write("GO\n")
            p.stdin.flush()
            for line in p.stdout:
                line = line.strip()
                if line.startswith("REFRESULT "):
                    res = json.loads(line[len("REFRESULT "):])
                    break
        if res is not None:
            res["clocks"] = clk.summary()
    try:
        p.stdin.close()
    except OSError:
        pass
    try:
        p.wait(timeout=120)
    except subprocess.TimeoutExpired:
        p.kill()
    log.close()
    got = torch.tensor([1 if res is not None else 0], dtype=torch.int64)
    if world > 1:
        torch.distributed.all_reduce(got, op=torch.distributed.ReduceOp.MIN)
    if int(got.item()) == 0:
        tail = open(log.name).read()[-600:].replace("\n", " | ")
        return {"failed": f"reference serving process ({'checked' if checked else 'unchecked'}) on rank {rank} "
                          f"gave no timings (rc {p.returncode}): {tail}"}
    for k in ("dev_ms", "wall_ms"):
        res[k] = max_over_ranks_cpu(res[k], world)
    res["alarms"] = int(sum_over_ranks_cpu(res["alarms"], world))
    return res


def max_over_ranks_cpu(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks_cpu(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64)
    torch.distributed.all_reduce(t)
    return float(t.item())


def run_reference(args, rank, world, local):
    if not os.path.isdir(os.path.join(_ref_dir(), "sdcguard")):
        return {"unavailable": "reference not installed in baseline/_ref"}
    checked = _ref_phase(args, rank, world, local, checked=True)
    if "failed" in checked:
        return {"unavailable": checked["failed"]}
    out = dict(checked)
    if not args.no_unchecked:
        un = _ref_phase(args, rank, world, local, checked=False)
        if "failed" not in un:
            out["unchecked_dev_ms"] = un["dev_ms"]
    out["false_alarms"] = checked["alarms"]
    return out


def main():
    args = parse()
    if args.ref_child:
        ref_child(args)
        return
    rank, world, local = dist_setup(use_gpu=args.impl == "ours")
    n = world
    res = run_ours(args, rank, world, local) if args.impl == "ours" else run_reference(args, rank, world, local)
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
                            "unit": "tokens/s (wall clock through generate(), prompts in, tokens out)",
                            "h2d_bytes_per_step": res.get("h2d_bytes", args.requests * 2048 * 8),
                            "d2h_bytes_per_step": args.requests * args.new_tokens * 8},
                    "false_alarms_clean_run": res["false_alarms"]}
            if "unchecked_dev_ms" in res:
                u = n * res["tokens_per_step"] / (res["unchecked_dev_ms"] / 1000.0)
                line["unchecked_value"] = round(u, 1)
                line["overhead_pct"] = round(100.0 * (u / tps - 1.0), 2)
            if args.impl == "reference":
                line["impl"] = "reference"
                line["path"] = (f"vllm {res.get('vllm')} LLM.generate + reference vllm_plugin (SDCGUARD=1, stock "
                                f"settings: linear-layer Triton check, attention recompute)")
                line["checked_layers"] = res.get("checked_layers")
            else:
                line["impl"] = "ours"
                line["gpu_launches"] = res["launches"]
                line["coverage"] = res["coverage"]
                if "campaign" in res:
                    line["detection"] = res["campaign"]
                for k in ("train", "tp", "ep", "pd"):
                    if k in res:
                        line[k] = res[k]
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
