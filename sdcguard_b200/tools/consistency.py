"""Does a server give the same answer along its different serving paths? Decode against prefill:

    python -m sdcguard_b200.tools.consistency http://127.0.0.1:8000 --probes 4 --tokens 24

A server reaches a token by different code depending on its state: decoded one at a time against the KV cache, or
computed in one prefill over the whole context. Each path has its own kernels (split-KV decode attention against
paged prefill attention, decode-sized GEMMs against prefill-sized ones) and bookkeeping, and a fault or bug can live
in one path only.

For each probe prompt P the server decodes t_1..t_n greedily, and three checks follow:

1. Cut points: P + t_1..t_k sent as a new prompt with max_tokens 1 must give t_(k+1) (position |P| + k computed by
   a prefill instead of a decode step).
2. Log-probabilities: P + t_1..t_n scored in one teacher-forced prefill (POST /v1/score, top-k log-probabilities of
   every position). At every position the decoded token must be the prefill's top token, or within MIN_GAP nats of
   it. A decoded token that the prefill ranks more than MIN_GAP nats below its top token, at a position where the
   prefill is sure of its top token (top two MIN_MARGIN nats apart), is a mismatch; a decoded token outside the
   prefill's top-k is a mismatch unless the k-th entry is within MIN_GAP of the top. Near ties between the top two
   prefill tokens are reported but do not count: rounding differences between the two paths can flip them.

3. Prefix cache (servers that keep one and export a hit counter, such as vLLM with this package's plugin): a long
   synthetic document plus a question is answered cold twice, each time under a salt of its own (vLLM's
   `cache_salt`: no cached block is shared), then answered again right after another question on the same document
   filled the cache under a shared salt. The server's hit counter must show the document's blocks read from the
   cache; the cached answer must then equal the cold one wherever the two cold answers agree with each other. A
   server that exports no prefix-cache counter gets NOT_APPLICABLE for this probe, which then takes no part in the
   verdict.

Verdicts: CONSISTENT (no mismatch), INCONSISTENT (a mismatch), INCONCLUSIVE (a request failed, the server does not
score, or the prefix-cache probe could not show a cache hit or got two different cold answers). CONSISTENT covers
these prompts and this server only. Exit 0 / 1 / 2. The report also gives the largest gap (nats) between a decoded
token and the prefill's top token over every compared position.

`judge_against(candidate, baseline)` judges a stack change: a candidate's mismatches count against it only when the
baseline run (same probes) was consistent, or when the candidate's largest gap exceeds the baseline's by more than
MIN_GAP; gaps the baseline shows as well are the serving paths' rounding on this model, not the change's doing.

Reference: src/sdcguard/consistency.py:1-45 (the decode-versus-prefill probe and its MIN_GAP / MIN_MARGIN lines),
:143 (the prefix-cache probe, which compares log-probabilities; this one compares the greedy tokens, which every
server returns, and needs the server's hit counter to judge at all).
"""
from __future__ import annotations

import argparse
import json
import random
import uuid
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


def _first_diff(a: list, b: list) -> Optional[int]:
    for i, (x, y) in enumerate(zip(a, b)):
        if x != y:
            return i
    return None if len(a) == len(b) else min(len(a), len(b))


def prefix_probe(base: str, documents: int = 4, doc_tokens: int = 256, question: int = 12, tokens: int = 16,
                 seed: int = 0, vocab: int = 1000, complete_salted: Callable = _client.complete_salted,
                 hits: Callable = _client.prefix_cache_hits) -> dict:
    """The prefix-cache probe (see the module docstring). `complete_salted(base, ids, n, salt)` answers under a
    cache salt; `hits(base)` reads the server's prefix-cache hit counter in tokens (None: no counter)."""
    if hits(base) is None:
        return {"verdict": "NOT_APPLICABLE", "why": "the server exports no prefix-cache hit counter", "cases": []}
    rng = random.Random(seed * 7919 + 17)
    cases, failed = [], []
    for d in range(documents):
        doc = [rng.randrange(vocab) for _ in range(doc_tokens)]
        qa = [rng.randrange(vocab) for _ in range(question)]
        qb = [rng.randrange(vocab) for _ in range(question)]
        try:
            cold = complete_salted(base, doc + qa, tokens, uuid.uuid4().hex)
            cold2 = complete_salted(base, doc + qa, tokens, uuid.uuid4().hex)
            shared = uuid.uuid4().hex
            h0 = hits(base)
            complete_salted(base, doc + qb, 1, shared)        # the document's blocks enter the cache
            warm = complete_salted(base, doc + qa, tokens, shared)
            h1 = hits(base)
        except Exception as e:  # noqa: BLE001  (a failed request makes the probe inconclusive)
            failed.append({"document": d, "error": str(e)[:300]})
            continue
        hit = None if h0 is None or h1 is None else (h1 - h0) >= doc_tokens // 2
        cases.append({"document": d, "prompt_tokens": doc_tokens + question, "cache_hit": hit,
                      "hit_tokens": None if h0 is None or h1 is None else h1 - h0,
                      "cold_repeat_first_difference": _first_diff(cold, cold2),
                      "cached_first_difference": _first_diff(cold, warm)})
    # a difference counts only where the cached path was shown taken and two cold answers agreed
    bad = [c for c in cases if c["cache_hit"] is True and c["cold_repeat_first_difference"] is None
           and c["cached_first_difference"] is not None]
    unsure = [c for c in cases if c["cache_hit"] is not True or c["cold_repeat_first_difference"] is not None]
    verdict = ("INCONSISTENT" if bad else "INCONCLUSIVE" if failed or not cases or unsure else "CONSISTENT")
    why = [f"document {c['document']}: the answer with its prefix read from the cache differs from the cold answer "
           f"at token {c['cached_first_difference']}, while two cold answers agreed" for c in bad]
    why += [f"document {c['document']}: " + ("no cache hit shown" if c["cache_hit"] is not True else
                                             "two cold answers differ (the server is not deterministic here)")
            for c in unsure]
    return {"verdict": verdict, "why": why, "cases": cases, "failed": failed,
            "probe_set": {"documents": documents, "doc_tokens": doc_tokens, "question": question, "tokens": tokens,
                          "seed": seed}}


def run(base: str, probes: int = 4, prompt: int = 48, tokens: int = 24, cuts=(1, 4, 8, 15), seed: int = 0,
        vocab: int = 1000, top_k: int = 5, complete: Callable = _client.complete,
        score: Optional[Callable] = _client.score, prefix: bool = True,
        complete_salted: Callable = _client.complete_salted, hits: Callable = _client.prefix_cache_hits) -> dict:
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
    decode_verdict = ("INCONSISTENT" if bad or lp_rows else
                      "INCONCLUSIVE" if failed or not (cut_rows or compared) else "CONSISTENT")
    pc = prefix_probe(base, seed=seed, vocab=vocab, complete_salted=complete_salted, hits=hits) if prefix else \
        {"verdict": "NOT_APPLICABLE", "why": "not run", "cases": []}
    pv = pc["verdict"]
    verdict = ("INCONSISTENT" if "INCONSISTENT" in (decode_verdict, pv) else
               "INCONCLUSIVE" if "INCONCLUSIVE" in (decode_verdict, pv) else "CONSISTENT")
    return {"schema": SCHEMA, "url": base, "verdict": verdict, "decode_verdict": decode_verdict, "prefix_cache": pc,
            "checks": len(cut_rows),
            "logprob_positions": compared, "largest_gap": round(largest, 4),
            "probe_set": {"probes": probes, "prompt": prompt, "tokens": tokens, "seed": seed}, "mismatches": bad,
            "logprob_mismatches": lp_rows, "near_ties": ties, "failed": failed,
            "scope": "these prompts and this server only"}


def judge_against(cand: dict, base: Optional[dict] = None) -> dict:
    """A candidate's consistency judged for a stack change (see the module docstring). The prefix-cache probe
    stands on its own: a cached answer must equal a cold one on any stack, whatever the baseline shows."""
    pc = cand.get("prefix_cache") or {}
    if pc.get("verdict") == "INCONSISTENT":
        return {"verdict": "INCONSISTENT", "why": ["prefix cache: " + (pc.get("why") or ["cached answer differs"])[0]]}
    if pc.get("verdict") == "INCONCLUSIVE":
        return {"verdict": "INCONCLUSIVE", "why": ["prefix cache: " + "; ".join(pc.get("why") or ["inconclusive"])]}
    v = cand.get("decode_verdict", cand.get("verdict"))
    if v not in ("CONSISTENT", "INCONSISTENT"):
        return {"verdict": "INCONCLUSIVE", "why": [f"the candidate's check was {v}"]}
    if v == "CONSISTENT":
        return {"verdict": "CONSISTENT", "why": ["decode matched prefill at every compared position"]}
    n = len(cand.get("mismatches") or []) + len(cand.get("logprob_mismatches") or [])
    if base is None:
        return {"verdict": "INCONSISTENT", "why": [f"{n} decode/prefill mismatches (no baseline run to compare)"]}
    if base.get("probe_set") != cand.get("probe_set"):
        return {"verdict": "INCONCLUSIVE", "why": ["the baseline ran other probes"]}
    if base.get("decode_verdict", base.get("verdict")) == "CONSISTENT":
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
    ap.add_argument("--no-prefix", action="store_true", help="skip the prefix-cache probe")
    ap.add_argument("--out")
    a = ap.parse_args(argv)
    r = run(a.url, a.probes, tokens=a.tokens, seed=a.seed, score=None if a.no_score else _client.score,
            prefix=not a.no_prefix)
    if a.out:
        with open(a.out, "w") as f:
            json.dump(r, f, indent=1)
    print(json.dumps({k: v for k, v in r.items() if k not in ("mismatches", "logprob_mismatches")}))
    return {"CONSISTENT": 0, "INCONSISTENT": 1}.get(r["verdict"], 2)


if __name__ == "__main__":
    raise SystemExit(main())
