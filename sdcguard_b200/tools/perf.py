"""How fast a server serves a fixed load, measured the same way on each side of a change.

    python -m sdcguard_b200.tools.perf http://127.0.0.1:8000 --out before.json      # the stack you run now
    ... change the stack, start it again ...
    python -m sdcguard_b200.tools.perf http://127.0.0.1:8000 --out after.json
    python -m sdcguard_b200.tools.perf --compare before.json after.json

The load is a fixed prompt set (token-id prompts of 32 to 256 tokens from a fixed seed, or one prompt per line of
--prompts-file), each a greedy completion of --max-tokens tokens, so every request asks for the same work on every
stack. Requests are streamed (`"stream": true`, server-sent events): per request the time to the first token, the
gaps between later tokens (inter-token latency) and the whole latency. --concurrency requests are in flight at a
time, after --warmup requests that are not measured, and the whole load runs --rounds times.

A request counts only when its stream ended with `[DONE]` and carried a usage record with a non-negative integer
completion_tokens; an error event, an HTTP error, a stream cut short or a malformed chunk make it an error (kept
with what was seen before it). Per round: output tokens per second (the tokens the server's usage records say it
generated, over the round's wall time), requests per second, and p50 / p99 of time to first token, inter-token gap
and latency. The report gives each round, the median over rounds and each metric's spread (max - min over median).

`compare` gives the candidate's medians against the baseline's, per metric: the change, whether it is better or worse
for that metric, and whether it is noise (no larger than the larger of NOISE_FLOOR and twice either side's spread).
Two runs of different loads, or a run with failed requests, are not compared (INCONCLUSIVE). Its verdict follows
output tokens per second: FASTER, SLOWER, SAME (within noise) or INCONCLUSIVE.

Reference: src/sdcguard/perf.py:1-25 (the fixed streamed load, per-request observations, medians and the
round-spread noise rule), `one_request` :112, `compare` :447.
"""
from __future__ import annotations

import argparse
import hashlib
import http.client
import json
import math
import queue
import random
import statistics
import threading
import time
from typing import Callable, Optional
from urllib.parse import urlparse

from . import _client

SCHEMA = "sdcguard.perf/1"
NOISE_FLOOR = 0.02
# metric -> which direction is better
METRICS = {"output_tokens_per_s": "higher", "requests_per_s": "higher",
           "ttft_p50_ms": "lower", "ttft_p99_ms": "lower", "itl_p50_ms": "lower", "itl_p99_ms": "lower",
           "latency_p50_ms": "lower", "latency_p99_ms": "lower"}


def default_load(n: int = 64, seed: int = 0, vocab: int = 1000, lo: int = 32, hi: int = 256) -> list:
    """The fixed prompt set: n token-id prompts of lo to hi tokens (the same on every run with the same seed)."""
    rng = random.Random(seed)
    return [[rng.randrange(1, vocab) for _ in range(rng.randrange(lo, hi + 1))] for _ in range(n)]


def load_digest(prompts: list) -> str:
    return hashlib.sha256(json.dumps(prompts, separators=(",", ":")).encode()).hexdigest()


def percentile(xs: list, q: float) -> Optional[float]:
    """Linear-interpolated q-quantile (q in [0, 1]) of a list; None when empty."""
    if not xs:
        return None
    s = sorted(xs)
    pos = q * (len(s) - 1)
    lo = int(math.floor(pos))
    hi = min(lo + 1, len(s) - 1)
    return s[lo] + (s[hi] - s[lo]) * (pos - lo)


class RequestFailed(RuntimeError):
    def __init__(self, message: str, seen: dict):
        super().__init__(message)
        self.seen = seen


def _strict_json(data: str):
    def no_constant(v):
        raise ValueError(f"non-finite JSON value {v}")

    def unique(pairs):
        out = {}
        for k, v in pairs:
            if k in out:
                raise ValueError(f"duplicate key {k!r}")
            out[k] = v
        return out
    obj = json.loads(data, parse_constant=no_constant, object_pairs_hook=unique)
    if not isinstance(obj, dict):
        raise ValueError("an event's data must be a JSON object")
    return obj


def stream_request(base: str, prompt, max_tokens: int, timeout: float = 600.0) -> dict:
    """One streamed greedy completion. Returns {ttft_s, gaps_s, latency_s, tokens, chunks}; raises RequestFailed
    (with the partial observation) unless the stream ends with [DONE] after a valid usage record."""
    u = urlparse(base)
    conn_cls = http.client.HTTPSConnection if u.scheme == "https" else http.client.HTTPConnection
    conn = conn_cls(u.hostname, u.port, timeout=timeout)
    seen = {"ttft_s": None, "gaps_s": [], "latency_s": None, "tokens": None, "chunks": 0, "done": False}
    t0 = time.perf_counter()
    last = None
    try:
        body = {"prompt": prompt, "max_tokens": max_tokens, "stream": True, "temperature": 0.0}
        conn.request("POST", (u.path.rstrip("/") or "") + "/v1/completions", body=json.dumps(body),
                     headers={"Content-Type": "application/json"})
        resp = conn.getresponse()
        if resp.status != 200:
            raise ValueError(f"HTTP {resp.status}: {resp.read()[:200]!r}")
        for raw in resp:
            line = raw.decode("utf-8").strip()
            if line.startswith("event:") and line[6:].strip() == "error":
                raise ValueError("the server sent an error event")
            if not line.startswith("data:"):
                continue
            data = line[5:].strip()
            if data == "[DONE]":
                seen["done"] = True
                break
            ev = _strict_json(data)
            if "error" in ev:
                raise ValueError(f"error in stream: {str(ev['error'])[:200]}")
            usage = ev.get("usage")
            if usage is not None:
                n = usage.get("completion_tokens") if isinstance(usage, dict) else None
                if type(n) is not int or n < 0:
                    raise ValueError("usage.completion_tokens is not a non-negative integer")
                if seen["tokens"] is not None and n != seen["tokens"]:
                    raise ValueError("two usage records disagree")
                seen["tokens"] = n
            choices = ev.get("choices") or []
            if not isinstance(choices, list):
                raise ValueError("choices is not a list")
            if any(isinstance(c, dict) and c.get("finish_reason") == "error" for c in choices):
                raise ValueError("a choice finished with an error")
            if any(isinstance(c, dict) and c.get("text") for c in choices):
                now = time.perf_counter()
                if seen["ttft_s"] is None:
                    seen["ttft_s"] = now - t0
                else:
                    seen["gaps_s"].append(now - last)
                last = now
                seen["chunks"] += 1
        if not seen["done"]:
            raise ValueError("the stream ended without [DONE]")
        if seen["tokens"] is None:
            raise ValueError("no usage record")
        if seen["chunks"] > seen["tokens"]:
            raise ValueError(f"{seen['chunks']} token chunks for {seen['tokens']} tokens in usage")
        return seen
    except Exception as e:  # noqa: BLE001  (every failure is the request's error, with what was seen)
        raise RequestFailed(f"{type(e).__name__}: {e}"[:300], seen) from e
    finally:
        seen["latency_s"] = time.perf_counter() - t0
        conn.close()


def _ms(x: Optional[float]) -> Optional[float]:
    return None if x is None else round(1000.0 * x, 3)


def run_round(base: str, prompts: list, concurrency: int, max_tokens: int,
              request: Callable = stream_request) -> dict:
    """Every prompt once, `concurrency` at a time; the round's throughput and latency percentiles."""
    todo: "queue.Queue" = queue.Queue()
    for i, p in enumerate(prompts):
        todo.put((i, p))
    done: list = []
    errors: list = []
    lock = threading.Lock()

    def worker():
        while True:
            try:
                i, p = todo.get_nowait()
            except queue.Empty:
                return
            try:
                r = request(base, p, max_tokens)
                with lock:
                    done.append(r)
            except RequestFailed as e:
                with lock:
                    errors.append({"request": i, "error": str(e), "seen": e.seen})
            except Exception as e:  # noqa: BLE001  (a request helper that raised something else)
                with lock:
                    errors.append({"request": i, "error": f"{type(e).__name__}: {e}"[:300]})

    t0 = time.perf_counter()
    th = [threading.Thread(target=worker, daemon=True) for _ in range(max(1, concurrency))]
    for t in th:
        t.start()
    for t in th:
        t.join()
    wall = time.perf_counter() - t0
    ttft = [r["ttft_s"] for r in done if r.get("ttft_s") is not None]
    gaps = [g for r in done for g in r.get("gaps_s") or []]
    lat = [r["latency_s"] for r in done if r.get("latency_s") is not None]
    toks = sum(r.get("tokens") or 0 for r in done)
    return {"requests": len(prompts), "completed": len(done), "errors": len(errors), "error_samples": errors[:3],
            "wall_s": round(wall, 4), "output_tokens": toks,
            "output_tokens_per_s": round(toks / wall, 3) if wall > 0 and done else None,
            "requests_per_s": round(len(done) / wall, 3) if wall > 0 and done else None,
            "ttft_p50_ms": _ms(percentile(ttft, 0.5)), "ttft_p99_ms": _ms(percentile(ttft, 0.99)),
            "itl_p50_ms": _ms(percentile(gaps, 0.5)), "itl_p99_ms": _ms(percentile(gaps, 0.99)),
            "latency_p50_ms": _ms(percentile(lat, 0.5)), "latency_p99_ms": _ms(percentile(lat, 0.99))}


def server_info(base: str) -> dict:
    """What the server says it is: its model (/v1/models) and, for this package's server, its stack record and
    whether its checks are on (/metrics)."""
    out: dict = {"model": None, "stack": None, "checks_on": None}
    try:
        data = json.loads(_client.get(base.rstrip("/") + "/v1/models", 10.0)).get("data") or []
        out["model"] = data[0].get("id") if data else None
    except Exception:  # noqa: BLE001  (a server without the endpoint)
        pass
    m = _client.scrape(base)
    if m:
        rows = m.get("sdcguard_stack_info{}") or []
        out["stack"] = rows[0][0] if rows else None
        if "sdcguard_protected" in m:
            out["checks_on"] = m["sdcguard_protected"] == 1
    return out


def _spread(vals: list) -> Optional[float]:
    if not vals or any(v is None for v in vals):
        return None
    med = statistics.median(vals)
    return (max(vals) - min(vals)) / med if med else None


def measure(base: str, prompts: Optional[list] = None, concurrency: int = 8, max_tokens: int = 32, rounds: int = 3,
            warmup: int = 4, request: Callable = stream_request, info: Callable = server_info) -> dict:
    prompts = default_load() if prompts is None else prompts
    if not prompts:
        raise ValueError("the load has no prompts")
    before = info(base)
    warm_errors = 0
    for p in prompts[:warmup]:
        try:
            request(base, p, max_tokens)
        except Exception:  # noqa: BLE001  (counted; a failing warm-up makes the run incomplete)
            warm_errors += 1
    rs = [run_round(base, prompts, concurrency, max_tokens, request) for _ in range(rounds)]
    after = info(base)
    med, spread = {}, {}
    for m in METRICS:
        vals = [r.get(m) for r in rs]
        ok = [v for v in vals if v is not None]
        med[m] = statistics.median(ok) if ok and len(ok) == len(vals) else None
        spread[m] = _spread(vals)
    why = []
    if warm_errors:
        why.append(f"{warm_errors} warm-up requests failed")
    if any(r["errors"] or r["completed"] != r["requests"] for r in rs):
        why.append("not every request of every round completed")
    if before.get("model") != after.get("model") or before.get("stack") != after.get("stack"):
        why.append("the server's model or stack record changed during the measurement")
    if med["output_tokens_per_s"] is None:
        why.append("no throughput was measured")
    return {"schema": SCHEMA, "url": base, "model": before.get("model"), "stack": before.get("stack"),
            "checks_on": before.get("checks_on"),
            "load": {"prompts": len(prompts), "prompts_sha256": load_digest(prompts), "concurrency": concurrency,
                     "max_tokens": max_tokens, "rounds": rounds, "warmup": warmup},
            "rounds": rs, "median": med, "spread": spread, "complete": not why, "why": why,
            "created": time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime())}


def compare(base: dict, cand: dict) -> dict:
    """The candidate's medians against the baseline's, per metric, with the noise rule of the module docstring."""
    why = []
    if base.get("load") != cand.get("load"):
        why.append("the two runs did not send the same load (prompts, concurrency, tokens, rounds)")
    for side, r in (("baseline", base), ("candidate", cand)):
        if not r.get("complete"):
            why.append(f"the {side} run is incomplete: " + "; ".join(r.get("why") or ["failed requests"]))
    out: dict = {"comparable": not why, "why": why, "metrics": {}, "models": [base.get("model"), cand.get("model")],
                 "verdict": "INCONCLUSIVE"}
    if why:
        return out
    for m, better in METRICS.items():
        b, c = base["median"].get(m), cand["median"].get(m)
        if b is None or c is None or b == 0:
            out["metrics"][m] = None
            continue
        change = (c - b) / b
        spreads = [s for s in (base["spread"].get(m), cand["spread"].get(m)) if s is not None]
        band = max([NOISE_FLOOR] + [2.0 * s for s in spreads])
        good = change > 0 if better == "higher" else change < 0
        out["metrics"][m] = {"baseline": b, "candidate": c, "change": round(change, 4),
                             "direction": "same" if change == 0 else "better" if good else "worse",
                             "noise_band": round(band, 4), "noise": abs(change) <= band}
    tp = out["metrics"].get("output_tokens_per_s")
    if tp is not None:
        out["verdict"] = "SAME" if tp["noise"] else "FASTER" if tp["change"] > 0 else "SLOWER"
        out["throughput_ratio"] = round(tp["candidate"] / tp["baseline"], 4)
    return out


def read_prompts(path: str) -> list:
    """One prompt per line: a JSON list of token ids, or text."""
    out = []
    with open(path) as f:
        for line in f:
            line = line.rstrip("\n")
            if not line.strip():
                continue
            if line.lstrip().startswith("["):
                out.append([int(t) for t in json.loads(line)])
            else:
                out.append(line)
    return out


def render(r: dict) -> str:
    if "metrics" in r:                           # a comparison
        lines = [f"perf comparison: {r['verdict']}"] + [f"  {w}" for w in r.get("why") or []]
        for m, x in r["metrics"].items():
            if x:
                lines.append(f"  {m}: {x['baseline']} -> {x['candidate']} ({x['change']:+.1%}, {x['direction']}"
                             + (", within noise" if x["noise"] else "") + ")")
        return "\n".join(lines)
    lines = [f"perf of {r['url']} (model {r.get('model')}, checks {'on' if r.get('checks_on') else 'off or unknown'})"
             f": {'complete' if r['complete'] else 'INCOMPLETE: ' + '; '.join(r['why'])}"]
    for m in METRICS:
        v, s = r["median"].get(m), r["spread"].get(m)
        lines.append(f"  {m}: {v}" + (f" (spread {s:.1%})" if s is not None else ""))
    return "\n".join(lines)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="sdcguard perf", description=__doc__.split("\n\n")[0])
    ap.add_argument("url", nargs="?")
    ap.add_argument("--prompts-file")
    ap.add_argument("--concurrency", type=int, default=8)
    ap.add_argument("--max-tokens", type=int, default=32)
    ap.add_argument("--rounds", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--out")
    ap.add_argument("--json", action="store_true")
    ap.add_argument("--compare", nargs=2, metavar=("BASELINE", "CANDIDATE"))
    a = ap.parse_args(argv)
    if a.compare:
        with open(a.compare[0]) as f0, open(a.compare[1]) as f1:
            r = compare(json.load(f0), json.load(f1))
        print(json.dumps(r, indent=1) if a.json else render(r))
        return 0 if r["comparable"] else 2
    if not a.url:
        ap.error("a server URL (or --compare) is required")
    r = measure(a.url, read_prompts(a.prompts_file) if a.prompts_file else None, a.concurrency, a.max_tokens,
                a.rounds, a.warmup)
    if a.out:
        with open(a.out, "w") as f:
            json.dump(r, f, indent=1)
    print(json.dumps(r, indent=1) if a.json else render(r))
    return 0 if r["complete"] else 2


if __name__ == "__main__":
    raise SystemExit(main())
