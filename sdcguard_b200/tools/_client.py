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


def complete(base: str, prompt, max_tokens: int, timeout: float = 600.0) -> list[int]:
    r = post(base.rstrip("/") + "/v1/completions", {"prompt": prompt, "max_tokens": max_tokens}, timeout)
    return r["choices"][0]["token_ids"]


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
