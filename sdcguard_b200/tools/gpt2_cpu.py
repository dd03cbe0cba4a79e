"""CPU fp32 detection benchmark: GPT-2 small (random init N(0, 0.02)), every nn.Linear checked by the fp32 ABFT
of `numerics.cpu_abft`, batch 4 x 128 token ids uniform over the vocabulary, seeded single-bit flips injected into
1% of the GEMM outputs (one flipped bit of one output element in 1% of the linear-layer calls). Reports the
detection rate (a detection = an alarm at the corrupted row and 128-column block), split by the flipped bit's
class and by whether the flip is larger than the fp32 rounding noise of its block, and the false alarms on the
clean calls.

    python -m sdcguard_b200.tools.gpt2_cpu --forwards 60 --rate 0.01 --seed 0 [--json]

Baseline for comparison: the reference has no fp32 check (0 of the 49 layers checkable); its bf16 check caught
47.9% of single-bit flips in bf16 GEMM outputs in the same kind of campaign on CPU.
"""
from __future__ import annotations

import argparse
import json
import math
import random
import time

import torch

from ..models.gpt2 import GPT2, GPT2Config
from ..numerics import abft
from ..numerics.cpu_abft import protect_cpu
from ..utils.inject import flip_bit_


def _bit_class(bit: int) -> str:
    return "sign" if bit == 31 else "exponent" if bit >= 23 else "mantissa_high" if bit >= 16 else "mantissa_low"


def run(forwards: int = 60, rate: float = 0.01, seed: int = 0, batch: int = 4, seq: int = 128,
        threads: int = 0, config: GPT2Config = GPT2Config()) -> dict:
    if threads:
        torch.set_num_threads(threads)
    torch.manual_seed(seed)
    model = GPT2(config, seed=seed).eval()
    rng = random.Random(seed)
    injections: list[dict] = []
    state_box: list = [None]

    def inject(y: torch.Tensor, name: str, call: int) -> None:
        if rng.random() >= rate:
            return
        flat = y.view(-1)
        i, bit = rng.randrange(flat.numel()), rng.randrange(32)
        old, new = flip_bit_(y, i, bit)
        n = y.shape[-1]
        row, col = divmod(i, n)
        d = {"layer": name, "call": call, "row": row, "block": col // abft.BLOCK, "bit": bit, "old": old,
             "new": new}
        injections.append(d)
        state_box[0].probes[call] = d          # the check stores its noise scale at (row, block) here

    g = torch.Generator().manual_seed(seed + 1)
    ids = [torch.randint(0, config.vocab, (batch, seq), generator=g) for _ in range(forwards)]
    # unchecked timing
    with torch.no_grad():
        model(ids[0])
        t0 = time.perf_counter()
        for x in ids[: min(5, forwards)]:
            model(x)
        t_plain = (time.perf_counter() - t0) / min(5, forwards)
    state = protect_cpu(model, inject=inject)
    state_box[0] = state
    # noise scale per injected block, to classify flips below the rounding noise
    t0 = time.perf_counter()
    with torch.no_grad():
        for x in ids:
            model(x)
    t_checked = (time.perf_counter() - t0) / forwards
    alarms = {(a["call"], a["row"], a["block"]): a for a in state.alarms}
    alarm_calls = {a["call"] for a in state.alarms}
    inj_calls = {d["call"] for d in injections}
    by_class: dict = {}
    caught = above = caught_above = 0
    for d in injections:
        hit = (d["call"], d["row"], d["block"]) in alarms
        delta = abs(d["new"] - d["old"]) if math.isfinite(d["new"]) else math.inf
        # above the noise: the flip moves the block sums by more than the alarm line (6 sigma of the block)
        big = delta > abft.Z_ALARM * d.get("sigma", 0.0)
        c = by_class.setdefault(_bit_class(d["bit"]), {"flips": 0, "caught": 0})
        c["flips"] += 1
        c["caught"] += int(hit)
        caught += int(hit)
        above += int(big)
        caught_above += int(hit and big)
    false_alarms = len([c for c in alarm_calls if c not in inj_calls])
    clean_worst = max((z for c, z in enumerate(state.call_z) if c not in inj_calls), default=0.0)
    return {"model": f"GPT-2 ({config.layers} layers, d={config.hidden}, {config.heads} heads, vocab {config.vocab}), "
                     "fp32, CPU",
            "batch": [batch, seq], "forwards": forwards, "linear_calls": state.calls,
            "checked_layers": len(state.worst), "checks": state.checks,
            "injection_rate": rate, "injected": len(injections), "caught": caught,
            "detection_rate": round(caught / max(1, len(injections)), 4),
            "flips_above_noise": above, "caught_above_noise": caught_above,
            "detection_rate_above_noise": round(caught_above / max(1, above), 4), "by_bit_class": by_class,
            "false_alarm_calls": false_alarms, "clean_calls": state.calls - len(inj_calls),
            "worst_clean_z": round(clean_worst, 4),
            "ms_per_forward_unchecked": round(1e3 * t_plain, 1), "ms_per_forward_checked": round(1e3 * t_checked, 1)}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m sdcguard_b200.tools.gpt2_cpu")
    ap.add_argument("--forwards", type=int, default=60)
    ap.add_argument("--rate", type=float, default=0.01)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--threads", type=int, default=0)
    ap.add_argument("--json", action="store_true")
    a = ap.parse_args(argv)
    r = run(a.forwards, a.rate, a.seed, threads=a.threads)
    print(json.dumps(r, indent=None if a.json else 1))
    return 0 if r["false_alarm_calls"] == 0 else 1


if __name__ == "__main__":
    raise SystemExit(main())
