"""Search a real (threaded) implementation for lifetime-breaking orderings, with no protocol model.

    from sdcguard_b200.lifetime import realsearch, toys
    res = realsearch.search(lambda: toys.ToyPush(fixed=False))
    print(realsearch.text(res))
    python -m sdcguard_b200.lifetime realsearch --toy push [--fixed]

The input is code instrumented with a `Probe`: its recording calls and its checkpoints (points where a thread could
legally be slow). The search knows nothing else about the protocol:

1. Baseline: run the system in its normal timing a few times, recording every checkpoint and event.
2. Footprint of each checkpoint: the regions the same thread touches after it, until its next checkpoint (the
   regions of its allocations, frees, consumes and of the operations it submits, lands or completes).
3. Candidate holds, each a single delay a stalled thread or late message could cause (nothing is fabricated):
   rule   from the ledger rules: hold the checkpoint until one of its regions is freed, reallocated, consumed by
          another request, or until an operation writing into it completes;
   flip   from the baseline: an event of another thread that came after the checkpoint; hold until it happens, so
          the observed order flips (with an empty footprint, any such event of another thread).
   Flips whose order never appeared in a baseline run go first.
4. Run each candidate on a fresh system; replay the recorded events through the ledger (`adapter.check`). A broken
   rule, or a run that did not finish (liveness), is a finding, reported with the hold that produced it; `replay`
   runs one candidate again to confirm it.

Reference: src/sdcguard/lifetime/realsearch.py:1-40 (baseline, footprints, rule and flip candidates, ranking,
`search`, `replay`, `text`).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, Optional

from . import adapter
from .probe import Hold, Probe

MAX_FLIPS_PER_CHECKPOINT = 8


@dataclass
class Candidate:
    thread: str
    name: str
    occurrence: int
    kind: str                  # "rule" or "flip"
    text: str
    until: Callable = field(repr=False)
    seen_in_baseline: bool = False

    def hold(self) -> Hold:
        return Hold(self.thread, self.name, self.occurrence, self.until, self.text)

    def key(self) -> tuple:
        return (self.thread, self.name, self.occurrence, self.text)


@dataclass
class RealFinding:
    rules: list
    candidate: str
    messages: list
    outcomes: dict
    finished: bool


@dataclass
class RealResult:
    findings: list
    tried: int
    baseline_runs: int
    baseline_clean: bool

    def as_dict(self) -> dict:
        return {"findings": [f.__dict__ for f in self.findings], "tried": self.tried,
                "baseline_runs": self.baseline_runs, "baseline_clean": self.baseline_clean}


def _run(make: Callable, hold: Optional[Hold] = None) -> tuple:
    p = Probe(hold)
    r = make().run(p)
    return p, r


def _regions_of(events: list, i: int, ops: dict) -> list:
    e = events[i]
    k = e["ev"]
    if k in ("alloc", "free", "share", "local_write", "consume"):
        return [tuple(e["region"])]
    if k == "submit":
        return [tuple(h[0]) for h in (e.get("src"), e.get("dst")) if h]
    if k in ("land", "complete", "stop") and e["op"] in ops:
        return ops[e["op"]]
    return []


def footprints(p: Probe) -> dict:
    """(thread, name, occurrence) -> (regions the thread touches after it, index of its first event)."""
    ev = p.events
    ops = {}
    for e in ev:
        if e["ev"] == "submit":
            ops[e["op"]] = [tuple(h[0]) for h in (e.get("src"), e.get("dst")) if h]
    out = {}
    cps = p.checkpoints
    for j, cp in enumerate(cps):
        nxt = next((c["at"] for c in cps[j + 1:] if c["thread"] == cp["thread"]), len(ev))
        regs = []
        for i in range(cp["at"], nxt):
            if ev[i].get("thread") == cp["thread"]:
                for r in _regions_of(ev, i, ops):
                    if r not in regs:
                        regs.append(r)
        out[(cp["thread"], cp["name"], cp["occurrence"])] = (regs, cp["at"])
    return out


def _until_event(pred: Callable[[dict], bool]) -> Callable:
    return lambda events, start: any(pred(e) for e in events[start:])


def _sig(e: dict) -> tuple:
    """An event's identity across runs: kind, thread, region (or the op's kind), owner / request."""
    reg = tuple(e["region"]) if "region" in e else None
    return (e["ev"], e.get("thread"), reg, e.get("kind"), e.get("owner"), e.get("request"))


def candidates(base: list) -> list[Candidate]:
    p0 = base[0][0]
    out, keys = [], set()

    def add(c: Candidate):
        if c.key() not in keys:
            keys.add(c.key())
            out.append(c)

    for (th, name, occ), (regs, at) in footprints(p0).items():
        for r in regs:
            rr = list(r)
            add(Candidate(th, name, occ, "rule", f"hold {th}@{name}#{occ} until {rr} is freed",
                          _until_event(lambda e, rr=rr: e["ev"] == "free" and e["region"] == rr)))
            add(Candidate(th, name, occ, "rule", f"hold {th}@{name}#{occ} until {rr} is reallocated",
                          _until_event(lambda e, rr=rr: e["ev"] == "alloc" and e["region"] == rr)))
            add(Candidate(th, name, occ, "rule", f"hold {th}@{name}#{occ} until another request consumes {rr}",
                          _until_event(lambda e, rr=rr, th=th: e["ev"] == "consume" and e["region"] == rr
                                       and e.get("thread") != th)))
            add(Candidate(th, name, occ, "rule", f"hold {th}@{name}#{occ} until a write into {rr} completes",
                          _until_event(lambda e, rr=rr, th=th: e["ev"] == "complete" and e.get("mark")
                                       and e["mark"][0] == rr and e.get("thread") != th)))
        n = 0
        for e in p0.events[at:]:
            if e.get("thread") == th:
                continue
            if regs and not any(x in regs for x in ([tuple(e["region"])] if "region" in e else [])
                                + [tuple(h[0]) for h in (e.get("src"), e.get("dst")) if h]):
                continue
            s = _sig(e)
            seen = any(_flipped_in(bp, th, name, occ, s) for bp, _ in base)
            add(Candidate(th, name, occ, "flip", f"hold {th}@{name}#{occ} until {s[1]} does {s[0]}"
                          + (f" on {list(s[2])}" if s[2] else "") + (f" ({s[3]})" if s[3] else ""),
                          _until_event(lambda x, s=s: _sig(x) == s), seen_in_baseline=seen))
            n += 1
            if n >= MAX_FLIPS_PER_CHECKPOINT:
                break
    return rank(out)


def _flipped_in(p: Probe, th: str, name: str, occ: int, sig: tuple) -> bool:
    """Did this baseline run already show the event before the checkpoint (the flipped order)?"""
    cp = next((c for c in p.checkpoints if (c["thread"], c["name"], c["occurrence"]) == (th, name, occ)), None)
    return cp is not None and any(_sig(e) == sig for e in p.events[:cp["at"]])


def rank(cands: list) -> list:
    """Rule holds, then flips never seen in a baseline, then the rest (stable within each group)."""
    return sorted(cands, key=lambda c: (0 if c.kind == "rule" else (1 if not c.seen_in_baseline else 2)))


def search(make: Callable, baseline_runs: int = 3, max_candidates: int = 64) -> RealResult:
    base = [_run(make) for _ in range(baseline_runs)]
    clean = all(not adapter.check(p.events)["violations"] and r["finished"] for p, r in base)
    findings, seen = [], set()
    cands = candidates(base)[:max_candidates]
    for c in cands:
        p, r = _run(make, c.hold())
        res = adapter.check(p.events)
        rules = sorted({v["rule"] for v in res["violations"]}) + ([] if r["finished"] else ["liveness"])
        if not rules:
            continue
        key = (tuple(rules), c.thread, c.name)
        if key in seen:
            continue
        seen.add(key)
        findings.append(RealFinding(rules, c.text, [v["message"] for v in res["violations"]][:5],
                                    r["outcomes"], r["finished"]))
    return RealResult(findings, len(cands), baseline_runs, clean)


def replay(make: Callable, cand: Candidate) -> dict:
    p, r = _run(make, cand.hold())
    return {"violations": adapter.check(p.events)["violations"], "finished": r["finished"],
            "outcomes": r["outcomes"], "events": p.events}


def text(res: RealResult) -> str:
    lines = [f"{res.tried} holds tried after {res.baseline_runs} baseline runs "
             f"({'clean' if res.baseline_clean else 'NOT clean'}); {len(res.findings)} finding(s)"]
    for f in res.findings:
        lines.append(f"  {'+'.join(f.rules)}: {f.candidate}")
        lines += [f"      {m}" for m in f.messages[:2]]
        lines.append(f"      outcomes {f.outcomes}, finished {f.finished}")
    return "\n".join(lines)
