"""The lifetime ledger: allocations of KV regions, their generations, outstanding operations, and four rules.

  region      a physical piece of KV memory, (pool, index)
  generation  a per-region counter that goes up at every allocation; a handle (region, generation) names one allocation
              and keeps naming it after the region is freed and reallocated
  owner       the request an allocation was made for; share() declares a permitted second consumer (a reused prefix)
  operation   an asynchronous access naming handles: "write" (into dst), "read" (src into dst), "load" (a host tier into
              dst). Outstanding from submit until it completes or the transport confirms it stopped; a cancel request
              alone does not stop it
  content     what a region holds, (owner, generation, label), set by local writes and by landed operations; consume()
              checks it, so a corruption is visible even when no rule caught its cause

Rules, checked as each event is recorded:
  R1 stale_handle       an operation submitted (or a descriptor accepted) for an allocation that is no longer current
  R2 reuse_outstanding  a region reallocated while an older operation that names it can still access it
  R3 consume_unready    a request consumes state that is not current, not its own or shared, still being written, or
                        holding someone else's content
  R4 stale_completion   a completion applied to an allocation its operation did not name

Allowed outcomes are not violations (a request failed or aborted after losing its lease, a rejected transfer, a free
with nothing outstanding). The ledger records and judges; it never decides what a server should do.

Reference: src/sdcguard/lifetime/ledger.py:1-36 (vocabulary and the four rules).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

RULES = {
    "R1": "stale_handle: an operation or descriptor used an allocation that is no longer current",
    "R2": "reuse_outstanding: a region was reallocated while an older operation could still access it",
    "R3": "consume_unready: state was consumed before it was current, ready and the consumer's own",
    "R4": "stale_completion: a completion was applied to an allocation its operation did not name",
}


@dataclass(frozen=True)
class Handle:
    region: tuple
    gen: int

    def __str__(self) -> str:
        return f"{self.region[0]}[{self.region[1]}]@{self.gen}"


@dataclass
class Region:
    gen: int = 0
    owner: Optional[str] = None
    sharers: set = field(default_factory=set)
    content: Optional[tuple] = None
    ready: bool = False


@dataclass
class Op:
    op_id: str
    kind: str
    src: Optional[Handle]
    dst: Optional[Handle]
    by: str
    payload: Optional[tuple] = None
    state: str = "outstanding"           # outstanding | completed | stopped
    cancel_requested: bool = False

    def names(self, region) -> bool:
        return any(h is not None and h.region == region for h in (self.src, self.dst))


@dataclass
class Violation:
    rule: str
    step: int
    message: str
    regions: tuple = ()
    ops: tuple = ()
    requests: tuple = ()


class Ledger:
    def __init__(self):
        self.regions: dict = {}
        self.ops: dict = {}
        self.violations: list = []
        self.events: list = []
        self.step = 0

    # ---------------------------------------------------------------- helpers
    def _reg(self, region) -> Region:
        return self.regions.setdefault(region, Region())

    def current(self, h: Handle) -> bool:
        r = self.regions.get(h.region)
        return r is not None and r.owner is not None and r.gen == h.gen

    def handle(self, region) -> Handle:
        return Handle(region, self._reg(region).gen)

    def _log(self, text: str, regions=(), ops=(), requests=()) -> None:
        self.events.append((self.step, text, tuple(regions), tuple(ops), tuple(requests)))

    def _violate(self, rule: str, msg: str, regions=(), ops=(), requests=()) -> None:
        self.violations.append(Violation(rule, self.step, msg, tuple(regions), tuple(ops), tuple(requests)))
        self._log(f"VIOLATION {rule}: {msg}", regions, ops, requests)

    # ---------------------------------------------------------------- events
    def alloc(self, region, owner: str) -> Handle:
        r = self._reg(region)
        live = [o for o in self.ops.values() if o.state == "outstanding" and o.names(region)]
        if live:
            self._violate("R2", f"{region} reallocated to {owner} while {', '.join(o.op_id for o in live)} can still "
                                f"access it", (region,), tuple(o.op_id for o in live), (owner,))
        r.gen += 1
        r.owner, r.sharers, r.ready = owner, set(), False
        h = Handle(region, r.gen)
        self._log(f"alloc {h} -> {owner}", (region,), (), (owner,))
        return h

    def free(self, h: Handle) -> None:
        r = self._reg(h.region)
        if r.gen == h.gen:
            r.owner, r.sharers, r.ready = None, set(), False
        self._log(f"free {h}", (h.region,))

    def share(self, h: Handle, request: str) -> None:
        if self.current(h):
            self.regions[h.region].sharers.add(request)
        self._log(f"share {h} with {request}", (h.region,), (), (request,))

    def local_write(self, h: Handle, by: str, label: str = "kv") -> None:
        r = self._reg(h.region)
        if self.current(h):
            r.content, r.ready = (r.owner, h.gen, label), True
        self._log(f"local write {h} by {by}", (h.region,), (), (by,))

    def submit(self, op_id: str, kind: str, by: str, src: Optional[Handle] = None, dst: Optional[Handle] = None,
               payload: Optional[tuple] = None) -> Op:
        for h in (src, dst):
            if h is not None and not self.current(h):
                self._violate("R1", f"{op_id} ({kind}) by {by} names {h}, not current", (h.region,), (op_id,), (by,))
        if payload is None and src is not None:
            payload = self._reg(src.region).content
        op = Op(op_id, kind, src, dst, by, payload)
        self.ops[op_id] = op
        self._log(f"submit {op_id} {kind} {src} -> {dst} by {by}",
                  tuple(h.region for h in (src, dst) if h is not None), (op_id,), (by,))
        return op

    def accept_descriptor(self, h: Handle, by: str) -> None:
        if not self.current(h):
            self._violate("R1", f"descriptor for {h} accepted by {by}, not current", (h.region,), (), (by,))
        self._log(f"accept descriptor {h} by {by}", (h.region,), (), (by,))

    def land(self, op_id: str) -> None:
        """The operation's data lands: a write / load sets the destination's content (whatever allocation the region
        holds now: that is exactly the corruption a late write causes)."""
        op = self.ops[op_id]
        if op.dst is not None and op.state == "outstanding":
            r = self._reg(op.dst.region)
            r.content = op.payload
        self._log(f"land {op_id}", (op.dst.region,) if op.dst else (), (op_id,))

    def complete(self, op_id: str, mark: Optional[Handle] = None) -> None:
        """The operation completed; `mark`: the allocation the completion is applied to (marks it ready)."""
        op = self.ops[op_id]
        op.state = "completed"
        if mark is not None:
            named = [h for h in (op.src, op.dst) if h is not None]
            if mark not in named:
                self._violate("R4", f"completion of {op_id} applied to {mark}, which it did not name ({', '.join(map(str, named))})",
                              (mark.region,), (op_id,))
            if self.current(mark):
                self.regions[mark.region].ready = True
        self._log(f"complete {op_id}" + (f" marks {mark}" if mark else ""), (mark.region,) if mark else (), (op_id,))

    def stop(self, op_id: str) -> None:
        self.ops[op_id].state = "stopped"
        self._log(f"stopped {op_id}", (), (op_id,))

    def cancel(self, op_id: str) -> None:
        self.ops[op_id].cancel_requested = True
        self._log(f"cancel requested {op_id}", (), (op_id,))

    def consume(self, h: Handle, request: str) -> None:
        r = self._reg(h.region)
        why = None
        if not self.current(h):
            why = f"{h} is not current"
        elif request != r.owner and request not in r.sharers:
            why = f"{h} belongs to {r.owner}"
        elif any(o.state == "outstanding" and o.dst is not None and o.dst.region == h.region
                 for o in self.ops.values()):
            why = f"{h} still has a transfer writing into it"
        elif not r.ready:
            why = f"{h} is not ready"
        elif r.content is None or r.content[1] != h.gen or (r.content[0] != request and request not in r.sharers
                                                              and r.content[0] != r.owner):
            why = f"{h} holds content {r.content}, not this allocation's"
        if why:
            self._violate("R3", f"{request} consumed {h}: {why}", (h.region,), (), (request,))
        self._log(f"consume {h} by {request}", (h.region,), (), (request,))
