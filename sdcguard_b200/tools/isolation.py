"""Cross-request influence probe: does what other requests are doing change a request's greedy output?

    python -m sdcguard_b200.tools.isolation http://127.0.0.1:8000 --probes 4 --primers 8

Each probe prompt is sent alone (twice: the server must repeat itself), then again while `primers` other requests
with different prompts and lengths run concurrently. With greedy decoding every token must match the solo answer.
A difference means the result depends on the batch it shared (batch-dependent kernels, a shared-state bug, or a
fault in one of the co-scheduled paths). Exit code 0 when every probe matched, 1 otherwise.

Reference: src/sdcguard/isolation.py (`primer_probe` :95).
"""
from __future__ import annotations

import argparse
import json
import random
import threading
from typing import Callable

from . import _client


def run(base: str, probes: int = 4, primers: int = 8, prompt: int = 64, tokens: int = 16, seed: int = 0,
        vocab: int = 1000, complete: Callable = _client.complete) -> dict:
    rng = random.Random(seed)
    rows = []
    for p in range(probes):
        ids = [rng.randrange(vocab) for _ in range(prompt)]
        solo = complete(base, ids, tokens)
        again = complete(base, ids, tokens)
        prim = [[rng.randrange(vocab) for _ in range(rng.randrange(8, 4 * prompt))] for _ in range(primers)]
        got: dict = {}

        def fire(i, x):
            got[i] = complete(base, x, tokens)

        th = [threading.Thread(target=fire, args=(i, x)) for i, x in enumerate(prim)]
        th.append(threading.Thread(target=fire, args=("probe", ids)))
        for t in th:
            t.start()
        for t in th:
            t.join()
        mixed = got.get("probe")
        rows.append({"probe": p, "repeat_matches": solo == again, "with_primers_matches": mixed == solo,
                     "first_difference": next((i for i, (a, b) in enumerate(zip(solo, mixed or [])) if a != b), None)})
    bad = [r for r in rows if not (r["repeat_matches"] and r["with_primers_matches"])]
    return {"url": base, "probes": rows, "verdict": "ISOLATED" if not bad else "INFLUENCED", "failed": len(bad)}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m sdcguard_b200.tools.isolation")
    ap.add_argument("url")
    ap.add_argument("--probes", type=int, default=4)
    ap.add_argument("--primers", type=int, default=8)
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)
    r = run(a.url, a.probes, a.primers, seed=a.seed)
    print(json.dumps(r))
    return 0 if r["verdict"] == "ISOLATED" else 1


if __name__ == "__main__":
    raise SystemExit(main())
