"""Delay-bounded exploration of a protocol model's event orderings, looking for one that breaks a ledger rule.

A model exposes, in each state, the actions that may happen next (a worker issuing a transfer, a transfer landing or
completing, a timeout, a request arriving); each names the resources it touches (its footprint). The default
schedule always takes the first enabled action (the model's unhurried order). Taking the k-th enabled action instead
costs k delays; with iterative deepening over the delay budget, the first schedule found for a rule has the fewest
delays. Only choices that conflict with the default action (intersecting footprints, or a footprint of "*") branch:
reordering independent actions cannot change what the ledger sees. States already seen with at least as much budget
left are not explored again.

A Finding is a broken rule with its schedule, reduced: each departure from the default order is undone in turn and
kept only if the violation needs it; the trace keeps the ledger events that touch the violation's regions,
operations and requests.

Reference: src/sdcguard/lifetime/explore.py:1-20 (delay bounding, conflict-only branching, reduction, causal trace).
"""
from __future__ import annotations

import copy
from dataclasses import dataclass, field
from typing import Callable

from .ledger import RULES


@dataclass(frozen=True)
class Action:
    label: str
    footprint: frozenset
    run: Callable = field(compare=False, repr=False, default=None)


def conflicts(a: Action, b: Action) -> bool:
    return "*" in a.footprint or "*" in b.footprint or bool(a.footprint & b.footprint)


@dataclass
class Finding:
    rule: str
    message: str
    schedule: list
    departures: list
    trace: list
    delays: int

    def as_dict(self) -> dict:
        return {"rule": self.rule, "rule_text": RULES[self.rule], "message": self.message, "delays": self.delays,
                "schedule": self.schedule, "departures": [list(d) for d in self.departures], "trace": self.trace}


@dataclass
class Result:
    model: str
    findings: list
    coverage: dict

    def as_dict(self) -> dict:
        return {"model": self.model, "findings": [f.as_dict() for f in self.findings], "coverage": self.coverage}


def _run(make: Callable, picks: dict, max_steps: int):
    """Replay: at step i take the action labelled picks[i] when enabled, else the default. Returns the model."""
    m = make()
    for i in range(max_steps):
        if m.ledger.violations or m.done():
            break
        acts = m.enabled()
        if not acts:
            break
        a = next((x for x in acts if x.label == picks.get(i)), acts[0])
        m.ledger.step = i
        a.run(m)
    return m


def _reduce(make: Callable, rule: str, departures: list, max_steps: int) -> tuple:
    deps = list(departures)
    i = 0
    while i < len(deps):
        trial = deps[:i] + deps[i + 1:]
        m = _run(make, {s: lab for s, lab, _ in trial}, max_steps)
        if m.ledger.violations and m.ledger.violations[0].rule == rule:
            deps = trial
        else:
            i += 1
    m = _run(make, {s: lab for s, lab, _ in deps}, max_steps)
    return deps, m


def _trace(m) -> list:
    v = m.ledger.violations[0]
    keys = set(v.regions) | set(v.ops) | set(v.requests)
    return [f"{s}: {t}" for s, t, regs, ops, reqs in m.ledger.events if keys & (set(regs) | set(ops) | set(reqs))]


def explore(make: Callable, budget: int = 2, max_steps: int = 60, max_states: int = 200_000) -> Result:
    """Search every schedule with at most `budget` delays (iterative deepening) for each rule's first violation."""
    found: dict = {}
    states = 0
    hit_bound = False
    name = make().name
    for b in range(budget + 1):
        seen: dict = {}
        stack = [(make(), [], [], b)]
        while stack:
            m, sched, deps, left = stack.pop()
            if m.ledger.violations:
                v = m.ledger.violations[0]
                if v.rule not in found:
                    found[v.rule] = (v.message, deps, b - left)
                continue
            if m.done() or len(sched) >= max_steps:
                hit_bound |= len(sched) >= max_steps and not m.done()
                continue
            acts = m.enabled()
            if not acts:
                continue
            sig = (m.signature(), len(sched) if getattr(m, "step_sensitive", False) else 0)
            if seen.get(sig, -1) >= left:
                continue
            seen[sig] = left
            states += 1
            if states > max_states:
                hit_bound = True
                stack.clear()
                break
            default = acts[0]
            choices = [(0, default)]
            for k, a in enumerate(acts[1:], 1):
                if k <= left and conflicts(a, default):
                    choices.append((k, a))
            for k, a in reversed(choices):
                m2 = copy.deepcopy(m) if len(choices) > 1 else m
                act = next(x for x in m2.enabled() if x.label == a.label)
                m2.ledger.step = len(sched)
                act.run(m2)
                stack.append((m2, sched + [a.label], deps + ([(len(sched), a.label, default.label)] if k else []),
                              left - k))
    findings = []
    for rule, (msg, deps, delays) in sorted(found.items()):
        rdeps, m = _reduce(make, rule, deps, max_steps)
        v = m.ledger.violations[0] if m.ledger.violations else None
        sched = [t for _, t, *_ in m.ledger.events]
        findings.append(Finding(rule, v.message if v else msg, sched, rdeps, _trace(m) if v else [], len(rdeps)))
    return Result(name, findings, {"budget": budget, "states": states, "bounds_hit": hit_bound,
                                   "assumptions": list(getattr(make(), "assumptions", ())),
                                   "not_covered": list(getattr(make(), "not_covered", ()))})
