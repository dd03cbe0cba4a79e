"""HTTP helpers shared by the server probes (ready, perf, isolation, consistency, qualify): completions requests and
Prometheus text parsing. Standard library only."""
from __future__ import annotations

import json
import re
import urllib.error
import urllib.request
from typing import Optional

_LINE = re.compile(r"^([a-zA-Z_:][\w:]*)(\{([^}]*)\})?\s+(\S+)")
_LAB = re.compile(r'(\w+)="([^"]*)"')


def get(url: str, timeout: float = 10.0) -> str:
    with urllib.request.urlopen(url, timeout=timeout) as r:
        return r.read().decode()


def post(url: str, body: dict, timeout: float = 600.0) -> dict:
    req = urllib.request.Request(url, data=json.dumps(body).encode(), headers={"Content-Type": "application/json"})
    with urllib.request.urlopen(req, timeout=timeout) as r:
        return json.loads(r.read().decode())


def complete(base: str, prompt, max_tokens: int, timeout: float = 600.0, extra: Optional[dict] = None) -> list[int]:
    """Greedy completion; `extra` adds fields to the request (vLLM's `cache_salt`, for one)."""
    r = post(base.rstrip("/") + "/v1/completions", {"prompt": prompt, "max_tokens": max_tokens, **(extra or {})},
             timeout)
    return r["choices"][0]["token_ids"]


def complete_salted(base: str, prompt, max_tokens: int, salt: str, timeout: float = 600.0) -> list[int]:
    """Greedy completion under a prefix-cache salt: requests with different salts share no cached blocks on a
    server that honours it (vLLM's `cache_salt`); a server without a prefix cache ignores the field."""
    return complete(base, prompt, max_tokens, timeout, extra={"cache_salt": salt})


def stream_cancel(base: str, prompt, max_tokens: int, timeout: float = 120.0) -> bool:
    """Start a streamed greedy completion and close the connection after its first event: the server is left to
    end a request whose client went away. Returns whether an event arrived before the close."""
    req = urllib.request.Request(base.rstrip("/") + "/v1/completions",
                                 data=json.dumps({"prompt": prompt, "max_tokens": max_tokens, "stream": True,
                                                  "temperature": 0.0}).encode(),
                                 headers={"Content-Type": "application/json"})
    with urllib.request.urlopen(req, timeout=timeout) as r:
        for raw in r:
            if raw.strip().startswith(b"data:"):
                return True
    return False


def prefix_cache_hits(base: str, timeout: float = 10.0) -> Optional[float]:
    """Tokens the server has read from its prefix cache so far (vLLM's `vllm:prefix_cache_hits` counter, summed
    over its labels), or None when the server exports no such counter."""
    m = scrape(base, timeout)
    if m is None:
        return None
    total, seen = 0.0, False
    for name, v in m.items():
        bare = name[:-2] if name.endswith("{}") else name
        if bare in ("vllm:prefix_cache_hits", "vllm:prefix_cache_hits_total"):
            seen = True
            total += sum(x for _, x in v) if isinstance(v, list) else v
    return total if seen else None


def score(base: str, prompt, top_k: int = 5, timeout: float = 600.0) -> dict:
    """Teacher-forced top-k log-probabilities of every position (POST /v1/score)."""
    return post(base.rstrip("/") + "/v1/score", {"prompt": prompt, "top_k": top_k}, timeout)


def parse_metrics(text: str) -> dict:
    """{name: value} for unlabelled samples; {name: [(labels, value), ...]} under name + '{}' for labelled ones."""
    out: dict = {}
    for line in text.splitlines():
        if not line or line.startswith("#"):
            continue
        m = _LINE.match(line)
        if not m:
            continue
        name, _, labels, val = m.groups()
        try:
            v = float(val)
        except ValueError:
            continue
        if labels is None:
            out[name] = v
        else:
            out.setdefault(name + "{}", []).append((dict(_LAB.findall(labels)), v))
    return out


def scrape(base: str, timeout: float = 10.0) -> Optional[dict]:
    try:
        return parse_metrics(get(base.rstrip("/") + "/metrics", timeout))
    except (urllib.error.URLError, OSError, ValueError):
        return None
