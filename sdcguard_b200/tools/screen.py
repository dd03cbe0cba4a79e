"""Workload screen of one GPU: a checked transformer served for a few minutes, the way the GPU will be used.

    python -m sdcguard_b200.tools.screen --size small --minutes 5 --out screen_out
    python -m sdcguard_b200.tools.screen --replay screen_out/evidence_r3.pt      # rerun a saved failing round
    python -m sdcguard_b200.tools.screen --size tiny --minutes 0 --simulate      # a demo: one flipped accumulator

Every round generates from a fixed set of random prompts with the checked decoder (every GEMM ABFT-checked on
tcgen05, attention / norm / rope / SwiGLU replay-checked on a sample of rows) and then generates again from the same
prompts: greedy decoding on this library's deterministic kernels must give the same tokens. A round fails when a
check alarms or the two runs differ; its prompts, seed, size, events and tokens are saved as evidence (`.pt`), and
`replay` reruns it to tell a reproducible fault (a defective unit) from a transient one. The report carries the GPU's
identity and telemetry before and after (nvidia-smi, read only) and is the input of `certify`.

Sizes (random-init weights): tiny (2 layers, d=256), small (8 layers, d=1024), 1b (16 layers, d=2048), 3b (28 layers,
d=3072). Exit code 0 pass, 1 fail, 2 could not run.

Reference: src/sdcguard/screen.py (ScreenModel sizes :49-94, evidence `_save_evidence` :280, `replay` :657).
"""
from __future__ import annotations

import argparse
import json
import os
import time
from typing import Optional

import torch

from ..utils.events import load_evidence, plain

from ..models.decoder import TINY, DecoderConfig
from .screen_ops import smi

SIZES = {
    "tiny": TINY,
    "small": DecoderConfig("screen-small", 8, 1024, 16, 8, 128, 3072, 32768, 1_000_000.0, 1e-6, True),
    "1b": DecoderConfig("screen-1b", 16, 2048, 16, 8, 128, 8192, 32768, 1_000_000.0, 1e-6, True),
    "3b": DecoderConfig("screen-3b", 28, 3072, 24, 8, 128, 8192, 32768, 1_000_000.0, 1e-6, True),
}
LOAD = {"tiny": (8, 96, 8), "small": (32, 512, 16), "1b": (32, 1024, 16), "3b": (32, 1024, 16)}  # batch, prompt, new


def _prompts(cfg, batch: int, plen: int, seed: int) -> tuple[torch.Tensor, list[int]]:
    g = torch.Generator().manual_seed(seed)
    lens = [int(x) for x in torch.randint(plen // 2, plen + 1, (batch,), generator=g)]
    return torch.randint(0, cfg.vocab, (batch, plen), generator=g).pin_memory(), lens


def _events(ev) -> list[dict]:
    return [{"detector": e.detector, "step": e.step, "detail": e.detail} for e in ev]


def run(device="cuda:0", size: str = "small", minutes: float = 2.0, seed: int = 0, out_dir: Optional[str] = None,
        simulate: bool = False, rounds: Optional[int] = None) -> dict:
    from ..serve.engine import LLMEngine
    dev = torch.device(device)
    cfg = SIZES[size]
    batch, plen, new = LOAD[size]
    t0 = time.time()
    rep = {"device": str(dev), "gpu": torch.cuda.get_device_name(dev), "size": size, "seed": seed,
           "minutes": minutes, "telemetry_before": smi(dev.index), "rounds": [], "simulated": simulate}
    eng = LLMEngine(cfg, device=dev, checked=True, num_blocks=batch * (-(-(plen + new) // 16)) + 8,
                    max_prefill_tokens=batch * plen, max_num_seqs=batch, sample_every=8,
                    max_model_len=plen + new, seed=seed)
    eng.guard.poll()
    deadline = t0 + 60 * minutes
    r = 0
    while True:
        prompts, lens = _prompts(cfg, batch, plen, seed * 1000 + r)
        if simulate and r == 0:
            eng.model.inject_next("L0.down", 3, 17, 1 << 30)
        a = eng.generate(prompts, lens, new)
        ev1 = eng.guard.poll()
        b = eng.generate(prompts, lens, new)
        ev2 = eng.guard.poll()
        mismatch = int((a != b).sum())
        row = {"round": r, "tokens": int(sum(lens) + batch * new) * 2, "alarms": len(ev1) + len(ev2),
               "mismatched_tokens": mismatch}
        if row["alarms"] or mismatch:
            row["events"] = _events(ev1 + ev2)
            if out_dir:
                os.makedirs(out_dir, exist_ok=True)
                path = os.path.join(out_dir, f"evidence_r{r}.pt")
                torch.save({"size": size, "seed": seed, "round": r, "prompts": prompts, "lens": lens, "new": new,
                            "tokens_a": a.cpu(), "tokens_b": b.cpu(), "events": plain(row["events"]), "gpu": plain(rep["gpu"]),
                            "simulated": simulate and r == 0}, path)
                row["evidence"] = path
        rep["rounds"].append(row)
        r += 1
        if (rounds is not None and r >= rounds) or (rounds is None and time.time() >= deadline):
            break
    cov = eng.guard.coverage_report()
    rep.update(checks=cov["checks"], unjudged=cov["unjudged"], worst_clean_z=cov["worst_clean_z"],
               tokens=sum(x["tokens"] for x in rep["rounds"]), seconds=round(time.time() - t0, 1),
               telemetry_after=smi(dev.index))
    bad = [x for x in rep["rounds"] if x["alarms"] or x["mismatched_tokens"]]
    rep["failed_rounds"] = [x["round"] for x in bad]
    rep["verdict"] = "FAIL" if bad else "PASS"
    if out_dir:
        os.makedirs(out_dir, exist_ok=True)
        with open(os.path.join(out_dir, "screen.json"), "w") as f:
            json.dump(rep, f, indent=1, default=str)
    return rep


def replay(path: str, device="cuda:0") -> dict:
    """Rerun a saved round twice on this device: reproducible (a check alarms or the tokens differ from the saved
    ones again) or not."""
    from ..serve.engine import LLMEngine
    ev = load_evidence(path)
    cfg = SIZES[ev["size"]]
    batch, plen, new = ev["prompts"].shape[0], ev["prompts"].shape[1], ev["new"]
    eng = LLMEngine(cfg, device=device, checked=True, num_blocks=batch * (-(-(plen + new) // 16)) + 8,
                    max_prefill_tokens=batch * plen, max_num_seqs=batch, sample_every=8,
                    max_model_len=plen + new, seed=ev["seed"])
    eng.guard.poll()
    outs, alarms = [], 0
    for _ in range(2):
        outs.append(eng.generate(ev["prompts"].pin_memory(), ev["lens"], new))
        alarms += len(eng.guard.poll())
    differs = [int((o != ev["tokens_a"]).sum()) for o in outs]
    repro = alarms > 0 or any(differs) or int((outs[0] != outs[1]).sum()) > 0
    return {"evidence": path, "alarms": alarms, "differs_from_saved": differs, "reproducible": repro,
            "classification": "reproducible (suspect a defective unit)" if repro else
            "not reproduced (transient, or injected)"}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m sdcguard_b200.tools.screen")
    ap.add_argument("--device", default="cuda:0")
    ap.add_argument("--size", default="small", choices=list(SIZES))
    ap.add_argument("--minutes", type=float, default=2.0)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--out", default=None)
    ap.add_argument("--simulate", action="store_true")
    ap.add_argument("--replay")
    a = ap.parse_args(argv)
    try:
        if a.replay:
            print(json.dumps(replay(a.replay, a.device)))
            return 0
        rep = run(a.device, a.size, a.minutes, a.seed, a.out, a.simulate)
    except Exception as e:  # noqa: BLE001
        print(json.dumps({"verdict": "error", "error": f"{type(e).__name__}: {e}"}))
        return 2
    print(json.dumps({k: rep[k] for k in ("verdict", "size", "checks", "tokens", "failed_rounds", "worst_clean_z",
                                          "seconds")}))
    return 0 if rep["verdict"] == "PASS" else 1


if __name__ == "__main__":
    raise SystemExit(main())
