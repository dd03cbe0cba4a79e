"""Lifetime events of a real engine: a JSONL sink the engine writes while it runs, and a checker that replays the
events through the ledger and reports every rule they break.

Event lines (one JSON object each; "region" is [pool, index], "gen" the allocation generation the engine saw):
  {"ev": "alloc", "region": r, "owner": req}          {"ev": "free", "region": r, "gen": g}
  {"ev": "share", "region": r, "gen": g, "request": req}
  {"ev": "local_write", "region": r, "gen": g, "by": req}
  {"ev": "submit", "op": id, "kind": "read"|"write"|"load", "by": who, "src": [r, g] | null, "dst": [r, g] | null}
  {"ev": "land", "op": id}   {"ev": "complete", "op": id, "mark": [r, g] | null}   {"ev": "stop", "op": id}
  {"ev": "consume", "region": r, "gen": g, "request": req}
  {"ev": "forward", "phase": "prefill"|"decode", "request": req, "regions": [[pool, idx, gen], ...],
   "positions": [first, last]}      (the block table one forward pass used for a request; not a ledger action)

`serve/pd.py` writes these for the prefill/decode path (producer pages, pulled pages, shared prefix pages, the decode
that consumes them, the frees). A model finding (models.py) is a candidate ordering; this is where a real run is held
to the same rules.

Reference: src/sdcguard/lifetime/adapter.py:46-246 (JSONL event sinks replayed through the ledger).
"""
from __future__ import annotations

import json
from typing import Iterable, Optional

from .ledger import Handle, Ledger


class EventSink:
    """Collects events (and appends them to a JSONL file when given); keeps the generation of every region so the
    engine can name handles."""

    def __init__(self, path: Optional[str] = None):
        self.events: list[dict] = []
        self.gen: dict = {}
        self._f = open(path, "a") if path else None
        self._ops = 0

    def _emit(self, ev: dict) -> None:
        self.events.append(ev)
        if self._f:
            self._f.write(json.dumps(ev) + "\n")
            self._f.flush()

    def ingest(self, events: list) -> None:
        """Events recorded by another process (a producer's page allocations), in order, before this one's own."""
        for e in events:
            if e["ev"] == "alloc":
                k = (e["region"][0], int(e["region"][1]))
                self.gen[k] = self.gen.get(k, 0) + 1
            self._emit(e)

    def handle(self, pool: str, idx: int) -> list:
        return [[pool, int(idx)], self.gen.get((pool, int(idx)), 0)]

    def alloc(self, pool: str, idx: int, owner: str) -> None:
        k = (pool, int(idx))
        self.gen[k] = self.gen.get(k, 0) + 1
        self._emit({"ev": "alloc", "region": [pool, int(idx)], "owner": owner})

    def free(self, pool: str, idx: int) -> None:
        r, g = self.handle(pool, idx)
        self._emit({"ev": "free", "region": r, "gen": g})

    def share(self, pool: str, idx: int, request: str) -> None:
        r, g = self.handle(pool, idx)
        self._emit({"ev": "share", "region": r, "gen": g, "request": request})

    def local_write(self, pool: str, idx: int, by: str) -> None:
        r, g = self.handle(pool, idx)
        self._emit({"ev": "local_write", "region": r, "gen": g, "by": by})

    def transfer(self, kind: str, by: str, src: Optional[tuple], dst: Optional[tuple],
                 src_gen: Optional[int] = None) -> str:
        """A synchronous transfer (submit, land, complete marking dst) between (pool, idx) pages. src_gen: the
        generation of the source allocation the transfer was planned for (default: the current one)."""
        self._ops += 1
        op = f"{kind}{self._ops}"
        s = self.handle(*src) if src else None
        if s is not None and src_gen is not None:
            s[1] = src_gen
        d = self.handle(*dst) if dst else None
        self._emit({"ev": "submit", "op": op, "kind": kind, "by": by, "src": s, "dst": d})
        self._emit({"ev": "land", "op": op})
        self._emit({"ev": "complete", "op": op, "mark": d})
        return op

    def consume(self, pool: str, idx: int, request: str) -> None:
        r, g = self.handle(pool, idx)
        self._emit({"ev": "consume", "region": r, "gen": g, "request": request})

    def forward(self, phase: str, request: str, pool: str, pages, first: int, last: int) -> None:
        """The block table a forward pass of `request` used (positions first..last), with each page's generation."""
        self._emit({"ev": "forward", "phase": phase, "request": request,
                    "regions": [[pool, int(p), self.gen.get((pool, int(p)), 0)] for p in pages],
                    "positions": [int(first), int(last)]})

    def close(self) -> None:
        if self._f:
            self._f.close()


def _h(x) -> Optional[Handle]:
    return None if x is None else Handle(tuple(x[0]), int(x[1]))


def check(events: Iterable[dict]) -> dict:
    """Replay events through a fresh ledger; returns the violations (rule, step, message) and counts."""
    led = Ledger()
    n = 0
    for i, e in enumerate(events):
        led.step = i
        n += 1
        k = e["ev"]
        if k == "alloc":
            led.alloc(tuple(e["region"]), e["owner"])
        elif k == "free":
            led.free(Handle(tuple(e["region"]), e["gen"]))
        elif k == "share":
            led.share(Handle(tuple(e["region"]), e["gen"]), e["request"])
        elif k == "local_write":
            led.local_write(Handle(tuple(e["region"]), e["gen"]), e.get("by", "?"))
        elif k == "submit":
            src, dst = _h(e.get("src")), _h(e.get("dst"))
            payload = None
            if dst is not None:
                if src is not None:       # a copy carries the source's data (whoever's it is now) to dst's allocation
                    sc = led.regions[src.region].content if src.region in led.regions else None
                    payload = (sc[0] if sc else None, dst.gen, sc[2] if sc else "kv")
                else:
                    payload = (led.regions[dst.region].owner if dst.region in led.regions else None, dst.gen, "kv")
            led.submit(e["op"], e["kind"], e.get("by", "?"), src=src, dst=dst, payload=payload)
        elif k == "land":
            led.land(e["op"])
        elif k == "complete":
            led.complete(e["op"], _h(e.get("mark")))
        elif k == "stop":
            led.stop(e["op"])
        elif k == "consume":
            led.consume(Handle(tuple(e["region"]), e["gen"]), e["request"])
        elif k == "forward":
            pass                          # judged by evidence.forward against the ownership the events record
        else:
            raise ValueError(f"unknown event {k!r} at line {i}")
    return {"events": n, "violations": [{"rule": v.rule, "step": v.step, "message": v.message}
                                        for v in led.violations]}


def load(path: str) -> list[dict]:
    with open(path) as f:
        return [json.loads(x) for x in f if x.strip()]
