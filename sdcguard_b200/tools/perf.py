"""Fixed-load throughput of a server: N concurrent clients, each sending requests of a fixed prompt length and
output length for a fixed time (or count), measured from the client side.

    python -m sdcguard_b200.tools.perf http://127.0.0.1:8000 --clients 16 --prompt 256 --tokens 32 --seconds 30

Reports requests/s, generated tokens/s, total tokens/s, latency percentiles (p50 / p90 / p99) and errors. Prompts are
random token ids from a fixed seed, so two servers (a baseline and a candidate) see the same load.

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


def compare(before: dict, after: dict) -> dict:
    """Candidate against baseline: throughput ratio and latency change."""
    r = after["total_tokens_per_s"] / before["total_tokens_per_s"] if before["total_tokens_per_s"] else None
    return {"throughput_ratio": round(r, 4) if r else None,
            "p50_latency_ratio": round(after["latency_ms"]["p50"] / before["latency_ms"]["p50"], 4)
            if before["latency_ms"]["p50"] and after["latency_ms"]["p50"] else None,
            "errors": [before["errors"], after["errors"]]}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m sdcguard_b200.tools.perf")
    ap.add_argument("url")
    ap.add_argument("--clients", type=int, default=8)
    ap.add_argument("--prompt", type=int, default=128)
    ap.add_argument("--tokens", type=int, default=16)
    ap.add_argument("--seconds", type=float, default=10.0)
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)
    r = run(a.url, a.clients, a.prompt, a.tokens, a.seconds, seed=a.seed)
    print(json.dumps(r))
    return 0 if r["requests"] and not r["errors"] else 1


if __name__ == "__main__":
    raise SystemExit(main())
