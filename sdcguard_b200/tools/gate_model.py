"""Output check of a serving-stack change: does the candidate stack give the model the same next-token distributions
as the trusted one, position by position, under teacher forcing?

    python -m sdcguard_b200.tools.gate_model ref --model tiny --out ref.pt                   # on the trusted stack
    python -m sdcguard_b200.tools.gate_model check ref.pt --out same.json                    # same stack: noise floor
    python -m sdcguard_b200.tools.gate_model check ref.pt --precision fp8 --out new.json --noise same.json

`ref` records greedy completions of a fixed prompt set and, over prompt + completion, the trusted stack's top-20
log-probabilities at every position (prefill path). `check` scores the same token sequences on the candidate stack
(teacher forcing: every position sees the same context, so one near-tie flip cannot make the rest diverge) and
compares per position:

  top-1 agreement   the candidate's most likely token equals the reference's
  KL                KL(reference || candidate) over the union of both top-20 sets, each renormalized over the union,
                    a token one side did not list taking that side's smallest listed probability (an upper bound)
  delta logprob     change of the recorded next token's log-probability

Verdict (starting lines; a same-stack run given as --noise moves them to 3 x what it measured):
  PASS  mean KL <= max(1e-3, 3 noise), top-1 >= 99% (or not significantly below the noise run's, z < 3), no prompt's
        mean KL above max(0.05, 3 x the noise run's worst)
  WARN  mean KL up to max(7e-3, 3 noise) or top-1 from 97% to 99%
  FAIL  anything further

Stacks are this library's engine configurations (precision bf16 / fp8, checked / unchecked, seed of the random-init
weights must match the reference's).

Reference: src/sdcguard/gate_model.py:1-40 (teacher forcing, the KL over the union of top-20 sets, verdict lines),
:124-280.
"""
from __future__ import annotations

import argparse
import json
import math
from typing import Optional

import torch

from ..utils.events import load_evidence

TOPK = 20


def _engine(model: str, precision: str, checked: bool, seed: int, device: str, max_len: int, n: int):
    from ..models.decoder import CONFIGS
    from ..serve.engine import LLMEngine
    cfg = CONFIGS[model]
    return LLMEngine(cfg, device=device, checked=checked, num_blocks=n * (-(-max_len // 16)) + 16,
                     max_prefill_tokens=max(n * max_len, max_len), max_num_seqs=n, max_model_len=max_len, seed=seed,
                     precision=precision)


def reference(model: str = "tiny", precision: str = "bf16", checked: bool = True, seed: int = 0, prompts: int = 16,
              prompt_len: int = 64, new: int = 32, device: str = "cuda:0", prompt_seed: int = 1234) -> dict:
    eng = _engine(model, precision, checked, seed, device, prompt_len + new, prompts)
    g = torch.Generator().manual_seed(prompt_seed)
    P = torch.randint(0, eng.cfg.vocab, (prompts, prompt_len), generator=g)
    comp = eng.generate(P.pin_memory(), [prompt_len] * prompts, new)
    seqs = [P[i].tolist() + comp[i].tolist() for i in range(prompts)]
    sc = eng.score(seqs, TOPK)
    return {"format": "sdcguard-b200-model-ref/1", "model": model, "seed": seed, "prompt_len": prompt_len,
            "stack": {"precision": precision, "checked": checked}, "seqs": seqs,
            "values": [v for v, _ in sc], "ids": [i for _, i in sc],
            "recorded_is_top1": float(sum((sc[k][1][prompt_len - 1:-1, 0] == torch.tensor(seqs[k][prompt_len:])).sum()
                                          for k in range(prompts)) / (prompts * new))}


def compare_position(rv: torch.Tensor, ri: torch.Tensor, cv: torch.Tensor, ci: torch.Tensor) -> float:
    """KL(ref || cand) over the union of both top-k id sets, each side renormalized over the union; an id a side did
    not list gets that side's smallest listed probability."""
    rp = dict(zip(ri.tolist(), rv.exp().tolist()))
    cp = dict(zip(ci.tolist(), cv.exp().tolist()))
    u = set(rp) | set(cp)
    rmin, cmin = min(rp.values()), min(cp.values())
    r = {t: rp.get(t, rmin) for t in u}
    c = {t: cp.get(t, cmin) for t in u}
    rs, cs = sum(r.values()), sum(c.values())
    return sum((r[t] / rs) * math.log((r[t] / rs) / (c[t] / cs)) for t in u if r[t] > 0)


def _against(ref: dict, sc: list) -> dict:
    """Per-position comparison of candidate scores sc[k] = (values, ids) with the reference's."""
    seqs = ref["seqs"]
    plens = ref.get("prompt_lens") or [ref["prompt_len"]] * len(seqs)
    per_prompt, agree, total, dlp = [], 0, 0, []
    for k, s in enumerate(seqs):
        rv, ri = torch.as_tensor(ref["values"][k]), torch.as_tensor(ref["ids"][k])
        cv, ci = torch.as_tensor(sc[k][0]), torch.as_tensor(sc[k][1])
        kls = []
        for p in range(plens[k] - 1, len(s) - 1):   # positions whose next token is a recorded completion token
            kls.append(compare_position(rv[p], ri[p], cv[p], ci[p]))
            agree += int(ri[p, 0] == ci[p, 0])
            total += 1
            tok = s[p + 1]
            rl = rv[p][ri[p] == tok]
            cl = cv[p][ci[p] == tok]
            if rl.numel() and cl.numel():
                dlp.append(float(cl[0] - rl[0]))
        per_prompt.append(sum(kls) / len(kls))
    return {"positions": total, "mean_kl": sum(per_prompt) / len(per_prompt), "top1_agreement": agree / total,
            "worst_prompt_kl": max(per_prompt), "mean_abs_delta_logprob": sum(map(abs, dlp)) / max(1, len(dlp))}


def check(ref: dict, precision: str = "bf16", checked: bool = True, device: str = "cuda:0",
          noise: Optional[dict] = None) -> dict:
    seqs = ref["seqs"]
    L = max(len(s) for s in seqs)
    eng = _engine(ref["model"], precision, checked, ref["seed"], device, L, len(seqs))
    sc = eng.score(seqs, TOPK)
    res = {"format": "sdcguard-b200-model-check/1", "stack": {"precision": precision, "checked": checked},
           "reference_stack": ref["stack"], **_against(ref, sc), "alarms": len(eng.guard.poll())}
    res.update(verdict(res, noise))
    return res


def reference_url(url: str, prompts: int = 8, prompt_len: int = 48, new: int = 16, prompt_seed: int = 1234,
                  vocab: int = 1000, complete=None, score=None) -> dict:
    """`reference` against a running server: greedy completions of a fixed prompt set, then the top-20
    log-probabilities of every position of prompt + completion from its /v1/score (one teacher-forced prefill)."""
    from . import _client
    complete, score = complete or _client.complete, score or _client.score
    g = torch.Generator().manual_seed(prompt_seed)
    P = torch.randint(1, vocab, (prompts, prompt_len), generator=g).tolist()
    seqs, vals, ids = [], [], []
    for p in P:
        s = p + list(complete(url, p, new))
        r = score(url, s, TOPK)
        seqs.append(s)
        vals.append(r["top_logprobs"])
        ids.append(r["top_ids"])
    return {"format": "sdcguard-b200-model-ref/1", "url": url, "prompt_len": prompt_len,
            "prompt_lens": [prompt_len] * prompts, "seqs": seqs, "values": vals, "ids": ids}


def check_url(ref: dict, url: str, noise: Optional[dict] = None, score=None) -> dict:
    """`check` against a running server: the reference's sequences scored by its /v1/score."""
    from . import _client
    score = score or _client.score
    sc = []
    for s in ref["seqs"]:
        r = score(url, s, TOPK)
        sc.append((r["top_logprobs"], r["top_ids"]))
    res = {"format": "sdcguard-b200-model-check/1", "url": url, **_against(ref, sc)}
    res.update(verdict(res, noise))
    return res


def verdict(r: dict, noise: Optional[dict] = None) -> dict:
    n_kl = noise["mean_kl"] if noise else 0.0
    n_worst = noise["worst_prompt_kl"] if noise else 0.0
    pass_kl, warn_kl = max(1e-3, 3 * n_kl), max(7e-3, 3 * n_kl)
    worst_pass, worst_fail = max(0.05, 3 * n_worst), max(0.1, 3 * n_worst)
    top1_ok = r["top1_agreement"] >= 0.99
    if noise and not top1_ok:            # not significantly below the noise run's agreement
        p1, p2, n = noise["top1_agreement"], r["top1_agreement"], r["positions"]
        p = (p1 + p2) / 2
        se = math.sqrt(max(p * (1 - p) * 2 / max(n, 1), 1e-12))
        top1_ok = (p1 - p2) / se < 3
    if r["mean_kl"] <= pass_kl and top1_ok and r["worst_prompt_kl"] <= worst_pass:
        v = "PASS"
    elif r["mean_kl"] <= warn_kl and r["top1_agreement"] >= 0.97 and r["worst_prompt_kl"] <= worst_fail:
        v = "WARN"
    else:
        v = "FAIL"
    return {"verdict": v, "lines": {"pass_kl": pass_kl, "warn_kl": warn_kl, "worst_prompt_pass": worst_pass,
                                    "worst_prompt_fail": worst_fail}}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m sdcguard_b200.tools.gate_model")
    sub = ap.add_subparsers(dest="cmd", required=True)
    r = sub.add_parser("ref")
    r.add_argument("--model", default="tiny")
    r.add_argument("--precision", default="bf16")
    r.add_argument("--unchecked", action="store_true")
    r.add_argument("--seed", type=int, default=0)
    r.add_argument("--prompts", type=int, default=16)
    r.add_argument("--out", required=True)
    c = sub.add_parser("check")
    c.add_argument("ref")
    c.add_argument("--precision", default="bf16")
    c.add_argument("--unchecked", action="store_true")
    c.add_argument("--noise")
    c.add_argument("--out")
    for p in (r, c):
        p.add_argument("--device", default="cuda:0")
    a = ap.parse_args(argv)
    if a.cmd == "ref":
        ref = reference(a.model, a.precision, not a.unchecked, a.seed, a.prompts, device=a.device)
        torch.save(ref, a.out)
        print(json.dumps({"out": a.out, "recorded_is_top1": ref["recorded_is_top1"]}))
        return 0
    ref = load_evidence(a.ref)
    noise = None
    if a.noise:
        with open(a.noise) as f:
            noise = json.load(f)
    res = check(ref, a.precision, not a.unchecked, a.device, noise)
    if a.out:
        with open(a.out, "w") as f:
            json.dump(res, f, indent=1)
    print(json.dumps(res))
    return {"PASS": 0, "WARN": 0}.get(res["verdict"], 1)


if __name__ == "__main__":
    raise SystemExit(main())
