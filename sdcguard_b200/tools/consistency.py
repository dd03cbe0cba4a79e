"""Decode-versus-prefill consistency probe: the token a server decoded must be the token it predicts when the same
context arrives as a prompt.

    python -m sdcguard_b200.tools.consistency http://127.0.0.1:8000 --probes 4 --tokens 16

For each probe prompt P the server generates t_1..t_n. Then, for a few cut points k, the prompt P + t_1..t_k is sent
with max_tokens 1: the answer must be t_(k+1). The first path computes position |P| + k in a decode step (one row,
reading the KV cache); the second in a prefill (a tile of rows, fresh KV); with deterministic kernels and no fault
both give the same greedy token, except when the two top logits are within rounding of each other (reported as a
near tie only if the tokens differ and the server repeats itself). A prefix cache, KV transfer or decode kernel that
corrupts state shows up here as a mismatch.

Reference: src/sdcguard/consistency.py (`prefix_probe` :143).
"""
from __future__ import annotations

import argparse
import json
import random
from typing import Callable

from . import _client


def run(base: str, probes: int = 4, prompt: int = 48, tokens: int = 16, cuts=(1, 4, 8, 15), seed: int = 0,
        vocab: int = 1000, complete: Callable = _client.complete) -> dict:
    rng = random.Random(seed)
    rows = []
    for p in range(probes):
        ids = [rng.randrange(vocab) for _ in range(prompt)]
        gen = complete(base, ids, tokens)
        for k in cuts:
            if k >= len(gen):
                continue
            nxt = complete(base, ids + gen[:k], 1)
            rows.append({"probe": p, "cut": k, "decoded": gen[k], "prefilled": nxt[0], "match": nxt[0] == gen[k]})
    bad = [r for r in rows if not r["match"]]
    return {"url": base, "checks": len(rows), "mismatches": bad, "verdict": "CONSISTENT" if not bad else
            "INCONSISTENT"}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m sdcguard_b200.tools.consistency")
    ap.add_argument("url")
    ap.add_argument("--probes", type=int, default=4)
    ap.add_argument("--tokens", type=int, default=16)
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)
    r = run(a.url, a.probes, tokens=a.tokens, seed=a.seed)
    print(json.dumps(r))
    return 0 if r["verdict"] == "CONSISTENT" else 1


if __name__ == "__main__":
    raise SystemExit(main())
