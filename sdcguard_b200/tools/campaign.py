"""Fault-injection campaign on the GPU paths: seeded single-bit flips, detection counted per target and per bit
class, plus the false alarms of the same checks on clean data.

Targets:
  * gemm_accumulator: one bit of one fp32 accumulator element of a checked GEMM, flipped inside the kernel
    before the check and the rounding (a compute fault). Detected when the ABFT score exceeds 6. Flips whose
    effect is below the fp32 rounding noise of the block (low mantissa bits) are reported separately as
    `below_noise`: the arithmetic identity cannot see them, and neither can any other tolerance check.
  * replay_rows: one bit of a stored output row that the replay sample covers (norm, activation, attention).
    The exact comparison sees every such flip.
  * spot_sampled_outputs: one bit of one stored GEMM output that the spot check samples, judged against that
    output's own bound (catches changes below its block's ABFT noise).

GEMM flips are also split by whether they change the stored bf16 output: a flip in a low fp32 mantissa bit that
the rounding to bf16 erases changes nothing any reader sees (`output_unchanged`), while `output_changing` counts
the flips a consumer of the layer would receive.

The reference's equivalent is its FaultInjector plus harm study (src/sdcguard/inject.py:198,
experiments/harm_study.py); its rounded-output check caught 47.9% of single-bit flips in bf16 outputs on the
same kind of campaign (measured on CPU from the reference, 240 trials).
"""
from __future__ import annotations

import math
import random

import torch

from ..numerics import abft
from ..ops import gemm, layers


def _bit_class(bit: int) -> str:
    if bit == 31:
        return "sign"
    if bit >= 23:
        return "exponent"
    if bit >= 16:
        return "mantissa_high"
    return "mantissa_low"


def quick(seed: int = 0, trials: int = 96, device="cuda") -> dict:
    rng = random.Random(seed)
    dev = torch.device(device)
    g = torch.Generator(device="cpu").manual_seed(seed)
    m, k, n = 512, 1024, 1024
    x = torch.randn(m, k, generator=g).to(dev).bfloat16()
    w = (torch.randn(n, k, generator=g) * 0.02).to(dev).bfloat16()
    cw = gemm.CheckedWeight(w)
    st = gemm.StateTable(dev, trials + 8)
    rs = gemm.row_sqnorm(x)
    out = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    # clean runs: false alarms
    clean_slot = st.add("clean", cw.nb)
    for _ in range(16):
        gemm.checked_linear(x, cw, st.state, clean_slot, row_sq=rs, out=out)
    ref = (x.float() @ w.float().t())
    by_class: dict = {}
    below_noise = {"flips": 0, "caught": 0}
    clean_out = out.clone()
    slots, stored = [], []
    for t in range(trials):
        row, col, bit = rng.randrange(m), rng.randrange(n), rng.randrange(32)
        s = st.add(f"inj{t}", cw.nb)
        gemm.checked_linear(x, cw, st.state, s, row_sq=rs, out=out, inject=(row, col, 1 << bit))
        stored.append(out[row, col].clone())        # the flipped element as the layer stored it
        slots.append((s, row, col, bit))
    torch.cuda.synchronize()
    changed = [bool((v.view(torch.int16) != clean_out[r, c].view(torch.int16)).item())
               for v, (_, r, c, _) in zip(stored, slots)]
    rows = st.read()
    clean = rows[clean_slot]
    # noise scale of each block, to classify flips that are below it
    prod_coef, out_coef = cw.prod_coef, cw.out_coef
    xn = rs.sqrt().cpu()
    wmax = cw.cs.wstat[:, :3].amax(1).cpu()
    blocks = ref.view(m, cw.nb, 128)
    cn = blocks.pow(2).sum(-1).sqrt().cpu()
    visible = {"flips": 0, "caught": 0}              # flips that change the stored bf16 output
    visible_hi = {"flips": 0, "caught": 0}           # ... among bits >= 16 (the bf16 part of the accumulator)
    invisible = {"flips": 0, "caught": 0}            # flips the rounding to bf16 erases (no stored value changes)
    for (s, row, col, bit), ch in zip(slots, changed):
        r = rows[s]
        caught = r["z"] > abft.Z_ALARM and r.get("row") == row and r.get("block") == col // 128
        v = float(ref[row, col])
        fv = torch.tensor([v], dtype=torch.float32).view(torch.int32)
        flipped = (fv ^ (1 << bit if bit < 31 else -(1 << 31))).view(torch.float32).item()
        delta = abs(flipped - v) if math.isfinite(flipped) else math.inf
        b = col // 128
        den = float(cn[row, b]) * out_coef + prod_coef * float(xn[row]) * float(wmax[b]) + abft.ABS_FLOOR
        cls = _bit_class(bit)
        c = by_class.setdefault(cls, {"flips": 0, "caught": 0, "above_noise": 0, "caught_above_noise": 0})
        c["flips"] += 1
        c["caught"] += int(caught)
        if delta > abft.Z_ALARM * den:
            c["above_noise"] += 1
            c["caught_above_noise"] += int(caught)
        else:
            below_noise["flips"] += 1
            below_noise["caught"] += int(caught)
        for bucket, member in ((visible, ch), (visible_hi, ch and bit >= 16), (invisible, not ch)):
            if member:
                bucket["flips"] += 1
                bucket["caught"] += int(caught)
    tot = sum(c["flips"] for c in by_class.values())
    cau = sum(c["caught"] for c in by_class.values())
    above = sum(c["above_noise"] for c in by_class.values())
    cabove = sum(c["caught_above_noise"] for c in by_class.values())

    # spot targets: one bit of one stored output that the spot check samples (bf16 bits: 0-6 mantissa, 7-14
    # exponent, 15 sign), judged against that output's own bound; and the clean samples for false alarms
    from ..ops import spot as spot_ops
    sched = spot_ops.SpotSchedule(n)
    sst = torch.zeros(2 * trials + 1, abft.STATE_COLS, dtype=torch.int64, device=dev)
    spot_rows_all = []
    for t in range(trials):
        rows_t, cols_t = sched.sample(m, t, dev)
        rr, cc = sched.rows(m, t), sched.columns(t)
        row, col, bit = rr[rng.randrange(len(rr))], cc[rng.randrange(len(cc))], rng.randrange(16)
        yy = clean_out.clone()
        yy.view(torch.int16)[row, col] ^= (1 << bit) if bit < 15 else -(1 << 15)
        spot_ops.spot_check(x, w, yy, rows_t, cols_t, sst[t])
        spot_ops.spot_check(x, w, clean_out, rows_t, cols_t, sst[trials + t])
        spot_rows_all.append((row, col, bit))
    torch.cuda.synchronize()
    sp = sst.cpu().tolist()
    spot_by = {}
    for t, (row, col, bit) in enumerate(spot_rows_all):
        d = abft.decode_state_row(sp[t])
        hit = d["z"] > abft.Z_ALARM and d["flat"] == row * n + col
        cls = "sign" if bit == 15 else ("exponent" if bit >= 7 else "mantissa")
        c = spot_by.setdefault(cls, {"flips": 0, "caught": 0})
        c["flips"] += 1
        c["caught"] += int(hit)
    spot_false = sum(1 for t in range(trials) if abft.decode_state_row(sp[trials + t])["z"] > abft.Z_ALARM)
    spot_caught = sum(c["caught"] for c in spot_by.values())

    # replay targets: flip one bit of a sampled row of a norm output and of an activation output
    hid = torch.randn(256, 1024, device=dev).bfloat16()
    wln = torch.ones(1024, device=dev, dtype=torch.bfloat16)
    y, _ = layers.add_rmsnorm(hid, wln, 1e-6)
    rows_s = torch.arange(0, 256, 64, dtype=torch.int32, device=dev)
    rst = torch.zeros(32, 4, dtype=torch.int64, device=dev)
    rep_caught, rep_n = 0, 0
    for t in range(16):
        yy = y.clone()
        r_i = int(rows_s[t % rows_s.numel()])
        yy.view(torch.int16)[r_i, rng.randrange(1024)] ^= (1 << rng.randrange(16))
        yr, _ = layers.add_rmsnorm(hid, wln, 1e-6, rows=rows_s)
        layers.compare_rows(yy, rows_s, yr, rst[t])
        rep_n += 1
    torch.cuda.synchronize()
    rep_caught = int(((rst[:16, 0] >> 32) == 0x7F800000).sum())
    clean_rep = torch.zeros(1, 4, dtype=torch.int64, device=dev)
    yr, _ = layers.add_rmsnorm(hid, wln, 1e-6, rows=rows_s)
    layers.compare_rows(y, rows_s, yr, clean_rep[0])
    torch.cuda.synchronize()
    return {
        "gemm_accumulator": {"flips": tot, "caught": cau, "rate": round(cau / max(1, tot), 4),
                             "above_noise": above, "caught_above_noise": cabove,
                             "rate_above_noise": round(cabove / max(1, above), 4),
                             "below_noise": below_noise, "by_bit_class": by_class,
                             "output_changing": dict(visible, rate=round(visible["caught"] / max(1, visible["flips"]), 4)),
                             "output_changing_bits_16_31": dict(
                                 visible_hi, rate=round(visible_hi["caught"] / max(1, visible_hi["flips"]), 4)),
                             "output_unchanged": invisible,
                             "clean_checks": 16, "clean_worst_z": round(clean["z"], 4),
                             "false_alarms": int(clean["z"] > abft.Z_ALARM)},
        "replay_rows": {"flips": rep_n, "caught": rep_caught, "rate": round(rep_caught / max(1, rep_n), 4),
                        "false_alarms": int(clean_rep[0, 0].item() != 0)},
        "spot_sampled_outputs": {"flips": trials, "caught": spot_caught, "rate": round(spot_caught / max(1, trials), 4),
                                 "by_bit_class": spot_by, "clean_checks": trials, "false_alarms": spot_false},
    }


def main(argv=None) -> int:
    """`sdcguard campaign [--seed S] [--trials N] [--device cuda:0] [--json]`: exit 0 when every flip above the
    noise was caught and the clean runs raised nothing, 1 otherwise."""
    import argparse
    import json
    ap = argparse.ArgumentParser(prog="sdcguard campaign")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--trials", type=int, default=96)
    ap.add_argument("--device", default="cuda:0")
    ap.add_argument("--json", action="store_true")
    a = ap.parse_args(argv)
    res = quick(a.seed, a.trials, a.device)
    g, r = res["gemm_accumulator"], res["replay_rows"]
    if a.json:
        print(json.dumps(res, sort_keys=True))
    else:
        print(f"gemm accumulator flips: {g['caught']}/{g['flips']} caught; above noise {g['caught_above_noise']}/"
              f"{g['above_noise']}; below noise {g['below_noise']['caught']}/{g['below_noise']['flips']}; "
              f"clean worst z {g['clean_worst_z']}, false alarms {g['false_alarms']}")
        for cls, c in sorted(g["by_bit_class"].items()):
            print(f"  {cls:14s} {c['caught']}/{c['flips']} (above noise {c['caught_above_noise']}/{c['above_noise']})")
        print(f"replayed-row flips: {r['caught']}/{r['flips']} caught; false alarms {r['false_alarms']}")
    ok = g["caught_above_noise"] == g["above_noise"] and not g["false_alarms"] and r["caught"] == r["flips"] \
        and not r["false_alarms"]
    return 0 if ok else 1


if __name__ == "__main__":
    raise SystemExit(main())
