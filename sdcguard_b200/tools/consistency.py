"""Does a server give the same answer along its different serving paths? Decode against prefill:

    python -m sdcguard_b200.tools.consistency http://127.0.0.1:8000 --probes 4 --tokens 24

A server reaches a token by different code depending on its state: decoded one at a time against the KV cache, or
computed in one prefill over the whole context. Each path has its own kernels (split-KV decode attention against
paged prefill attention, decode-sized GEMMs against prefill-sized ones) and bookkeeping, and a fault or bug can live
in one path only.

For each probe prompt P the server decodes t_1..t_n greedily. Two checks:

1. Cut points: P + t_1..t_k sent as a new prompt with max_tokens 1 must give t_(k+1) (position |P| + k computed by
   a prefill instead of a decode step).
2. Log-probabilities: P + t_1..t_n scored in one teacher-forced prefill (POST /v1/score, top-k log-probabilities of
   every position). At every position the decoded token must be the prefill's top token, or within MIN_GAP nats of
   it. A decoded token that the prefill ranks more than MIN_GAP nats below its top token, at a position where the
   prefill is sure of its top token (top two MIN_MARGIN nats apart), is a mismatch; a decoded token outside the
   prefill's top-k is a mismatch unless the k-th entry is within MIN_GAP of the top. Near ties between the top two
   prefill tokens are reported but do not count: rounding differences between the two paths can flip them.

Verdicts: CONSISTENT (no mismatch), INCONSISTENT (a mismatch), INCONCLUSIVE (a request failed or the server does not
score). CONSISTENT covers these prompts and this server only. Exit 0 / 1 / 2. The report also gives the largest gap
(nats) between a decoded token and the prefill's top token over every compared position.

`judge_against(candidate, baseline)` judges a stack change: a candidate's mismatches count against it only when the
baseline run (same probes) was consistent, or when the candidate's largest gap exceeds the baseline's by more than
MIN_GAP; gaps the baseline shows as well are the serving paths' rounding on this model, not the change's doing.

Reference: src/sdcguard/consistency.py:1-45 (the decode-versus-prefill probe and its MIN_GAP / MIN_MARGIN lines; the
prefix-cache probe applies to servers with a prefix cache, which this package's engine does not keep).
"""
from __future__ import annotations

import argparse
import json
import random
from typing import Callable, Optional

from . import _client

SCHEMA = "sdcguard.consistency/1"
MIN_GAP = 0.5       # nats
MIN_MARGIN = 1.0    # nats


def logprob_check(prompt_len: int, gen: list, scored: dict) -> dict:
    """Compare decoded tokens with the teacher-forced prefill distribution of the same context."""
    vals, ids = scored["top_logprobs"], scored["top_ids"]
    rows, ties, compared, largest = [], 0, 0, 0.0
    for j, tok in enumerate(gen):
        pos = prompt_len + j - 1                     # the position whose distribution predicts gen[j]
        if pos < 0 or pos >= len(vals):
            continue
        v, i = vals[pos], ids[pos]
        compared += 1
        top, margin = v[0], (v[0] - v[1]) if len(v) > 1 else float("inf")
        if tok == i[0]:
            continue
        largest = max(largest, top - v[i.index(tok)] if tok in i else top - v[-1])
        if margin < MIN_GAP:
            ties += 1
            continue
        if tok in i:
            gap = top - v[i.index(tok)]
        else:
            gap = top - v[-1]                        # at least this far below the top
            if gap < MIN_GAP:
                ties += 1
                continue
        if gap > MIN_GAP and margin >= MIN_MARGIN:
            rows.append({"generated_index": j, "decoded": tok, "prefill_top": i[0], "gap_nats": round(gap, 4),
                         "prefill_margin_nats": round(margin, 4)})
        else:
            ties += 1
    return {"mismatches": rows, "near_ties": ties, "compared": compared, "largest_gap": round(largest, 4)}


def run(base: str, probes: int = 4, prompt: int = 48, tokens: int = 24, cuts=(1, 4, 8, 15), seed: int = 0,
        vocab: int = 1000, top_k: int = 5, complete: Callable = _client.complete,
        score: Optional[Callable] = _client.score) -> dict:
    rng = random.Random(seed)
    cut_rows, lp_rows, ties, failed, compared, largest = [], [], 0, [], 0, 0.0
    for p in range(probes):
        ids = [rng.randrange(vocab) for _ in range(prompt)]
        try:
            gen = complete(base, ids, tokens)
            for k in cuts:
                if k >= len(gen):
                    continue
                nxt = complete(base, ids + gen[:k], 1)
                cut_rows.append({"probe": p, "cut": k, "decoded": gen[k], "prefilled": nxt[0],
                                 "match": nxt[0] == gen[k]})
            if score is not None:
                lp = logprob_check(len(ids), gen, score(base, ids + gen, top_k))
                ties += lp["near_ties"]
                compared += lp["compared"]
                largest = max(largest, lp["largest_gap"])
                lp_rows += [dict(r, probe=p) for r in lp["mismatches"]]
        except Exception as e:  # noqa: BLE001  (a failed request makes the verdict inconclusive)
            failed.append({"probe": p, "error": str(e)[:300]})
    bad = [r for r in cut_rows if not r["match"]]
    verdict = ("INCONSISTENT" if bad or lp_rows else
               "INCONCLUSIVE" if failed or not (cut_rows or compared) else "CONSISTENT")
    return {"schema": SCHEMA, "url": base, "verdict": verdict, "checks": len(cut_rows),
            "logprob_positions": compared, "largest_gap": round(largest, 4),
            "probe_set": {"probes": probes, "prompt": prompt, "tokens": tokens, "seed": seed}, "mismatches": bad,
            "logprob_mismatches": lp_rows, "near_ties": ties, "failed": failed,
            "scope": "these prompts and this server only"}


def judge_against(cand: dict, base: Optional[dict] = None) -> dict:
    """A candidate's consistency judged for a stack change (see the module docstring)."""
    v = cand.get("verdict")
    if v not in ("CONSISTENT", "INCONSISTENT"):
        return {"verdict": "INCONCLUSIVE", "why": [f"the candidate's check was {v}"]}
    if v == "CONSISTENT":
        return {"verdict": "CONSISTENT", "why": ["decode matched prefill at every compared position"]}
    n = len(cand.get("mismatches") or []) + len(cand.get("logprob_mismatches") or [])
    if base is None:
        return {"verdict": "INCONSISTENT", "why": [f"{n} decode/prefill mismatches (no baseline run to compare)"]}
    if base.get("probe_set") != cand.get("probe_set"):
        return {"verdict": "INCONCLUSIVE", "why": ["the baseline ran other probes"]}
    if base.get("verdict") == "CONSISTENT":
        return {"verdict": "INCONSISTENT", "why": [f"{n} decode/prefill mismatches; the baseline had none"]}
    g_c, g_b = cand.get("largest_gap") or 0.0, base.get("largest_gap") or 0.0
    if g_c > g_b + MIN_GAP:
        return {"verdict": "INCONSISTENT", "why": [f"largest decode/prefill gap {g_c:.3f} nats against the "
                                                   f"baseline's {g_b:.3f}"]}
    return {"verdict": "CONSISTENT", "why": [f"the baseline shows the same decode/prefill gaps (largest {g_b:.3f} "
                                             f"nats; the candidate's {g_c:.3f}): not introduced by the change"]}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="sdcguard consistency")
    ap.add_argument("url")
    ap.add_argument("--probes", type=int, default=4)
    ap.add_argument("--tokens", type=int, default=24)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-score", action="store_true", help="cut points only (for servers without /v1/score)")
    ap.add_argument("--out")
    a = ap.parse_args(argv)
    r = run(a.url, a.probes, tokens=a.tokens, seed=a.seed, score=None if a.no_score else _client.score)
    if a.out:
        with open(a.out, "w") as f:
            json.dump(r, f, indent=1)
    print(json.dumps({k: v for k, v in r.items() if k not in ("mismatches", "logprob_mismatches")}))
    return {"CONSISTENT": 0, "INCONSISTENT": 1}.get(r["verdict"], 2)


if __name__ == "__main__":
    raise SystemExit(main())
