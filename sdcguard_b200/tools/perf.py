"""Fixed-load throughput of a server: N concurrent clients, each sending requests of a fixed prompt length and
output length for a fixed time (or count), measured from the client side.

    python -m sdcguard_b200.tools.perf http://127.0.0.1:8000 --clients 16 --prompt 256 --tokens 32 --seconds 30

Reports requests/s, generated tokens/s, total tokens/s, latency percentiles (p50 / p90 / p99) and errors. Prompts are
random token ids from a fixed seed, so two servers (a baseline and a candidate) see the same load. `measure` runs a
warm-up (not counted) and several rounds of the load and reports each round's throughput with their mean and
spread; `compare` judges a candidate against a baseline with that spread:

    python -m sdcguard_b200.tools.perf URL --rounds 3 --warmup 5 --out cand.json
    python -m sdcguard_b200.tools.perf --compare base.json cand.json    # FASTER / SLOWER / SAME / INCONCLUSIVE

A difference counts only when it exceeds both NOISE_FLOOR (2 %) and twice the larger relative spread (max - min
over mean) of the two measurements' rounds; a measurement with errors, or with fewer than two rounds, makes the
comparison INCONCLUSIVE.

Reference: src/sdcguard/perf.py (`one_request` :112; fixed-load throughput for the stack-change decision).
"""
from __future__ import annotations

import argparse
import json
import random
import statistics
import threading
import time
from typing import Callable

from . import _client


def run(base: str, clients: int = 8, prompt: int = 128, tokens: int = 16, seconds: float = 10.0,
        max_requests: int = 0, seed: int = 0, vocab: int = 1000, complete: Callable = _client.complete) -> dict:
    lat, errs = [], []
    lock = threading.Lock()
    stop = time.time() + seconds
    count = [0]

    def client(i: int):
        rng = random.Random(seed * 1000 + i)
        while time.time() < stop:
            with lock:
                if max_requests and count[0] >= max_requests:
                    return
                count[0] += 1
            ids = [rng.randrange(vocab) for _ in range(prompt)]
            t0 = time.perf_counter()
            try:
                out = complete(base, ids, tokens)
                ok = len(out) == tokens
            except Exception as e:  # noqa: BLE001  (counted)
                with lock:
                    errs.append(str(e)[:200])
                continue
            with lock:
                (lat if ok else errs).append(time.perf_counter() - t0 if ok else "short reply")

    t0 = time.perf_counter()
    th = [threading.Thread(target=client, args=(i,)) for i in range(clients)]
    for t in th:
        t.start()
    for t in th:
        t.join()
    wall = time.perf_counter() - t0
    n = len(lat)
    q = sorted(lat)

    def pct(p):
        return round(q[min(n - 1, int(p * n))] * 1e3, 1) if n else None

    return {"url": base, "clients": clients, "prompt": prompt, "tokens": tokens, "seconds": round(wall, 2),
            "requests": n, "errors": len(errs), "first_errors": errs[:3], "requests_per_s": round(n / wall, 2),
            "generated_tokens_per_s": round(n * tokens / wall, 1),
            "total_tokens_per_s": round(n * (tokens + prompt) / wall, 1),
            "latency_ms": {"p50": pct(0.5), "p90": pct(0.9), "p99": pct(0.99),
                           "mean": round(statistics.fmean(lat) * 1e3, 1) if n else None}}


NOISE_FLOOR = 0.02


def measure(base: str, rounds: int = 3, warmup: float = 5.0, **kw) -> dict:
    """A warm-up (not counted) and `rounds` rounds of the fixed load; each round's result and their summary."""
    if warmup > 0:
        run(base, **{**kw, "seconds": warmup})
    rs = [run(base, **kw) for _ in range(max(1, rounds))]
    tps = [r["total_tokens_per_s"] for r in rs]
    mean = statistics.fmean(tps)
    return {"url": base, "rounds": rs, "total_tokens_per_s": round(mean, 1),
            "spread": round((max(tps) - min(tps)) / mean, 4) if mean else None,
            "errors": sum(r["errors"] for r in rs), "latency_ms": rs[-1]["latency_ms"]}


def compare(before: dict, after: dict) -> dict:
    """Candidate against baseline: throughput ratio, latency change and, for measurements with rounds, a verdict
    that a difference within the rounds' spread cannot carry."""
    r = after["total_tokens_per_s"] / before["total_tokens_per_s"] if before["total_tokens_per_s"] else None
    out = {"throughput_ratio": round(r, 4) if r else None,
           "p50_latency_ratio": round(after["latency_ms"]["p50"] / before["latency_ms"]["p50"], 4)
           if before["latency_ms"]["p50"] and after["latency_ms"]["p50"] else None,
           "errors": [before["errors"], after["errors"]]}
    spreads = [m.get("spread") for m in (before, after)]
    if r is None or before["errors"] or after["errors"] or any(s is None for s in spreads) or \
            min(len(before.get("rounds", [])), len(after.get("rounds", []))) < 2:
        out["verdict"] = "INCONCLUSIVE"
        return out
    line = max(NOISE_FLOOR, 2 * max(spreads))
    out["noise_line"] = round(line, 4)
    out["verdict"] = "FASTER" if r > 1 + line else "SLOWER" if r < 1 - line else "SAME"
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="sdcguard perf")
    ap.add_argument("url", nargs="?")
    ap.add_argument("--clients", type=int, default=8)
    ap.add_argument("--prompt", type=int, default=128)
    ap.add_argument("--tokens", type=int, default=16)
    ap.add_argument("--seconds", type=float, default=10.0)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--rounds", type=int, default=1)
    ap.add_argument("--warmup", type=float, default=0.0)
    ap.add_argument("--out")
    ap.add_argument("--compare", nargs=2, metavar=("BASE", "CAND"))
    a = ap.parse_args(argv)
    if a.compare:
        with open(a.compare[0]) as f:
            b = json.load(f)
        with open(a.compare[1]) as f:
            c = json.load(f)
        res = compare(b, c)
        print(json.dumps(res))
        return {"FASTER": 0, "SAME": 0, "SLOWER": 1}.get(res.get("verdict"), 2)
    if not a.url:
        ap.error("a server URL (or --compare BASE CAND)")
    kw = dict(clients=a.clients, prompt=a.prompt, tokens=a.tokens, seconds=a.seconds, seed=a.seed)
    r = measure(a.url, a.rounds, a.warmup, **kw) if a.rounds > 1 or a.warmup > 0 else run(a.url, **kw)
    if a.out:
        with open(a.out, "w") as f:
            json.dump(r, f, indent=1)
    print(json.dumps({k: v for k, v in r.items() if k != "rounds"}))
    return 0 if r.get("total_tokens_per_s") and not r["errors"] else 1


if __name__ == "__main__":
    raise SystemExit(main())
