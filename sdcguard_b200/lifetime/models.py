"""Protocol models of KV-state lifetime, each in a buggy and a fixed variant. The explorer finds the buggy variants'
bad orderings with no bug-specific script: a model states the protocol (who allocates, publishes, transfers, times out,
frees and consumes) and the explorer chooses the order.

pd-abort      prefill pushes KV into a block the decode side allocated; the decode side aborts a request whose prefill
              is late. buggy: frees the block at once, so the next request gets it while the old write is in flight.
              fixed: sends the abort to the prefill side and reclaims only after the answer (no write issued, or every
              issued write completed or stopped). release-timeout: the fixed handshake with a drain timeout that frees
              anyway (a liveness fallback a timeout cannot make safe).
pd-lease      decode pulls KV from blocks the prefill side holds under a lease. buggy: the lease expires and the
              producer reuses its blocks while the read is delayed. fixed: the consumer pins before reading; a pinned
              lease never expires and a late pin is answered "expired" (the request fails: an allowed outcome).
pd-notify     transfer-done notifications are matched to requests by request id on a channel unordered with control
              messages. buggy: a retried request reuses the id, and a late notification of the aborted transfer marks
              the new allocation ready before its own transfer lands. fixed: notifications carry the transfer id and
              the allocation generation; stale ones are dropped.
offload-load  a prefix-cache hit loads KV from a host tier into a GPU block on a load stream. buggy: the forward pass
              starts once the load is issued. fixed: it waits for the load's completion.

Each model states its assumptions and what it does not cover. A model finding is a candidate ordering; a server
finding needs the same ordering driven in the real implementation (adapter.py checks recorded events).

Reference: src/sdcguard/lifetime/models.py:1-40 (the four families and their variants).
"""
from __future__ import annotations

from .explore import Action
from .ledger import Ledger

CLOCK = frozenset({"*"})


class _Model:
    key = ""
    VARIANTS = ("buggy", "fixed")
    assumptions: tuple = ()
    not_covered: tuple = ()

    def __init__(self, variant: str = "buggy"):
        if variant not in self.VARIANTS:
            raise ValueError(f"variant must be one of {self.VARIANTS}")
        self.variant = variant
        self.name = f"{self.key}:{variant}"
        self.ledger = Ledger()
        self.s: dict = {}
        self.h: dict = {}

    def signature(self):
        led = self.ledger
        regs = tuple(sorted((k, r.gen, r.owner, tuple(sorted(r.sharers)), r.content, r.ready)
                            for k, r in led.regions.items()))
        ops = tuple(sorted((k, o.state, o.cancel_requested) for k, o in led.ops.items()))
        return tuple(sorted(self.s.items())), regs, ops

    def act(self, label, footprint, fn):
        return Action(label, frozenset(footprint), fn)


class PDAbort(_Model):
    key = "pd-abort"
    VARIANTS = ("buggy", "fixed", "release-timeout")
    assumptions = ("the transport delivers a write at most once", "the prefill side knows which writes it issued",
                   "one decode block, so a new request reuses it")
    not_covered = ("partial writes", "several prefill workers")
    B = ("decode", 0)

    def enabled(self):
        s, B, acts = self.s, self.B, []
        led = self.ledger
        w = led.ops.get("w1")
        if not s.get("a1"):
            acts.append(self.act("D alloc r1", {B, "r1"}, lambda m: m._alloc1()))
            return acts
        if s.get("a1") and not s.get("sub") and not s.get("abort"):
            acts.append(self.act("P write r1 -> block", {B, "w1", "r1"}, lambda m: m._submit()))
        if w and w.state == "outstanding" and not s.get("landed"):
            acts.append(self.act("net write lands", {B, "w1"}, lambda m: m._land()))
        if w and w.state == "outstanding" and s.get("landed"):
            acts.append(self.act("net write completes", {B, "w1", "r1"}, lambda m: m._complete()))
        if s.get("ready1") and not s.get("done1") and not s.get("abort"):
            acts.append(self.act("D consume r1", {B, "r1"}, lambda m: m._consume1()))
        if s.get("done1") and not s.get("abort") and not s.get("freed"):
            acts.append(self.act("D free r1", {B, "r1"}, lambda m: m._free()))
        if s.get("freed") and not s.get("a2"):
            acts.append(self.act("C r2 arrives, D alloc r2", {B, "r2"}, lambda m: m._alloc2()))
        if s.get("a2") and not s.get("w2"):
            acts.append(self.act("D local write r2", {B, "r2"}, lambda m: m._write2()))
        if s.get("w2") and not s.get("done2"):
            acts.append(self.act("D consume r2", {B, "r2"}, lambda m: m._consume2()))
        # the decode side's patience runs out (a delay to choose: the normal order finishes first)
        if s.get("a1") and not s.get("done1") and not s.get("abort"):
            acts.append(self.act("clock: r1 prefill timeout, D aborts r1", CLOCK, lambda m: m._abort()))
        if s.get("abort") and self.variant != "buggy" and not s.get("answered"):
            if w and w.state == "outstanding":
                acts.append(self.act("P stops its write (transport confirms)", {"w1", B}, lambda m: m._stop()))
            if not w or w.state != "outstanding":
                acts.append(self.act("P answers abort: no write in flight", {"r1", B}, lambda m: m._answer()))
            if self.variant == "release-timeout" and not s.get("freed"):
                acts.append(self.act("clock: drain timeout, D frees anyway", CLOCK, lambda m: m._free_anyway()))
        if s.get("abort") and self.variant != "buggy" and s.get("answered") and not s.get("freed"):
            acts.append(self.act("D reclaims r1 after the answer", {B, "r1"}, lambda m: m._free()))
        return acts

    def done(self):
        return bool(self.s.get("done2"))

    def _alloc1(self):
        self.h["r1"] = self.ledger.alloc(self.B, "r1")
        self.s["a1"] = True

    def _submit(self):
        self.ledger.submit("w1", "write", "prefill", dst=self.h["r1"], payload=("r1", self.h["r1"].gen, "kv"))
        self.s["sub"] = True

    def _land(self):
        self.ledger.land("w1")
        self.s["landed"] = True

    def _complete(self):
        self.ledger.complete("w1", self.h["r1"])
        self.s["ready1"] = True

    def _consume1(self):
        self.ledger.consume(self.h["r1"], "r1")
        self.s["done1"] = True

    def _free(self):
        self.ledger.free(self.h["r1"])
        self.s["freed"] = True

    def _free_anyway(self):
        self._free()
        self.s["timeout_free"] = True

    def _abort(self):
        self.s["abort"] = True
        self.s["done1"] = True               # the request is gone (an allowed outcome)
        if self.variant == "buggy":
            self._free()

    def _stop(self):
        self.ledger.stop("w1")

    def _answer(self):
        self.s["answered"] = True

    def _alloc2(self):
        self.h["r2"] = self.ledger.alloc(self.B, "r2")
        self.s["a2"] = True

    def _write2(self):
        self.ledger.local_write(self.h["r2"], "r2")
        self.s["w2"] = True

    def _consume2(self):
        self.ledger.consume(self.h["r2"], "r2")
        self.s["done2"] = True


class PDLease(_Model):
    key = "pd-lease"
    assumptions = ("one producer block, reused by the next request", "reads are atomic once started")
    not_covered = ("lease renewal", "several consumers of one block")
    B = ("prefill", 0)

    def enabled(self):
        s, B, acts = self.s, self.B, []
        led = self.ledger
        rd = led.ops.get("rd")
        if not s.get("a1"):
            return [self.act("P alloc + write r1 (leased)", {B, "r1"}, lambda m: m._alloc1())]
        if self.variant == "fixed" and not s.get("pinned") and not s.get("failed") and not s.get("rd") and \
                not s.get("expired"):
            acts.append(self.act("C pins the lease", {B, "r1"}, lambda m: m._pin()))
        can_read = self.variant == "buggy" or s.get("pinned")
        if can_read and not s.get("rd") and not s.get("failed"):
            acts.append(self.act("C submits read", {B, "rd", "r1"}, lambda m: m._read()))
        if rd and rd.state == "outstanding":
            acts.append(self.act("net read completes", {B, "rd"}, lambda m: m._read_done()))
        if s.get("got") and not s.get("used"):
            acts.append(self.act("C consumes its copy", {"r1", ("decode", 0)}, lambda m: m._use()))
        if s.get("used") and not s.get("released"):
            acts.append(self.act("C releases the lease", {B, "r1"}, lambda m: m._release()))
        if s.get("released") and not s.get("a2"):
            acts.append(self.act("P alloc r2", {B, "r2"}, lambda m: m._alloc2()))
        if not s.get("released") and not s.get("expired") and not s.get("pinned"):
            acts.append(self.act("clock: lease expires, P reuses the block", CLOCK, lambda m: m._expire()))
        if self.variant == "fixed" and s.get("expired") and not s.get("failed") and not s.get("rd"):
            acts.append(self.act("C's late pin answered expired: request fails", {"r1"}, lambda m: m._fail()))
        return acts

    def done(self):
        return bool(self.s.get("a2") and (self.s.get("used") or self.s.get("failed")))

    def _alloc1(self):
        self.h["r1"] = self.ledger.alloc(self.B, "r1")
        self.ledger.local_write(self.h["r1"], "r1")
        self.s["a1"] = True

    def _pin(self):
        self.s["pinned"] = True

    def _read(self):
        self.h["dst"] = self.ledger.alloc(("decode", 0), "r1")
        self.ledger.submit("rd", "read", "decode", src=self.h["r1"], dst=self.h["dst"])
        self.s["rd"] = True

    def _read_done(self):
        self.ledger.land("rd")
        self.ledger.complete("rd", self.h["dst"])
        self.s["got"] = True

    def _use(self):
        self.ledger.consume(self.h["dst"], "r1")
        self.s["used"] = True

    def _release(self):
        self.ledger.free(self.h["r1"])
        self.s["released"] = True

    def _expire(self):
        self.s["expired"] = True
        self.ledger.free(self.h["r1"])
        self.s["released"] = True

    def _fail(self):
        self.s["failed"] = True

    def _alloc2(self):
        self.h["r2"] = self.ledger.alloc(self.B, "r2")
        self.ledger.local_write(self.h["r2"], "r2")
        self.s["a2"] = True


class PDNotify(_Model):
    key = "pd-notify"
    assumptions = ("notifications and control messages are unordered with respect to each other",
                   "a retried request keeps its request id")
    not_covered = ("duplicate notifications of one transfer",)
    B = ("decode", 0)

    def enabled(self):
        s, B, acts = self.s, self.B, []
        if not s.get("a1"):
            return [self.act("D alloc r (first try), P writes t1", {B, "t1"}, lambda m: m._start1())]
        t1 = self.ledger.ops.get("t1")
        if t1 and t1.state == "outstanding" and not s.get("landed1"):
            acts.append(self.act("net t1 lands", {B, "t1"}, lambda m: m._land1()))
        if s.get("landed1") and not s.get("notified1") and not s.get("retried"):
            acts.append(self.act("notify t1 done (request r)", {B, "t1", "r"}, lambda m: m._notify1()))
        if s.get("ready") and not s.get("consumed"):
            acts.append(self.act("D consumes r", {B, "r"}, lambda m: m._consume()))
        if not s.get("retried") and not s.get("consumed"):
            acts.append(self.act("clock: r times out; abort, retry r into a new allocation, P writes t2", CLOCK,
                                 lambda m: m._retry()))
        if s.get("retried"):
            t2 = self.ledger.ops.get("t2")
            if t1 and t1.state == "outstanding" and not s.get("late1"):
                acts.append(self.act("late notify t1 done (request r)", {B, "t1", "r"}, lambda m: m._late1()))
            if t2 and t2.state == "outstanding" and not s.get("landed2"):
                acts.append(self.act("net t2 lands", {B, "t2"}, lambda m: m._land2()))
            if s.get("landed2") and t2.state == "outstanding":
                acts.append(self.act("notify t2 done (request r)", {B, "t2", "r"}, lambda m: m._notify2()))
        return acts

    def done(self):
        return bool(self.s.get("consumed"))

    def _start1(self):
        self.h["a1"] = self.ledger.alloc(self.B, "r")
        self.ledger.submit("t1", "write", "prefill", dst=self.h["a1"], payload=("r", self.h["a1"].gen, "kv"))
        self.s["a1"] = True

    def _land1(self):
        self.ledger.land("t1")
        self.s["landed1"] = True

    def _notify1(self):
        self.ledger.complete("t1", self.h["a1"])
        self.s["notified1"] = True
        self.s["ready"] = True

    def _consume(self):
        h = self.h.get("a2", self.h["a1"])
        self.ledger.consume(h, "r")
        self.s["consumed"] = True

    def _retry(self):
        self.s["retried"] = True
        self.s["ready"] = False
        # the abort does not stop t1: it may still land and notify
        self.ledger.free(self.h["a1"])
        self.h["a2"] = self.ledger.alloc(("decode", 1), "r")
        self.ledger.submit("t2", "write", "prefill", dst=self.h["a2"], payload=("r", self.h["a2"].gen, "kv"))

    def _late1(self):
        self.s["late1"] = True
        if self.variant == "buggy":          # matched by request id: marks the current allocation of r ready
            self.ledger.complete("t1", self.h["a2"])
            self.s["ready"] = True
        else:                                # carries t1 and generation: stale, dropped
            self.ledger.complete("t1")

    def _land2(self):
        self.ledger.land("t2")
        self.s["landed2"] = True

    def _notify2(self):
        self.ledger.complete("t2", self.h["a2"])
        self.s["ready"] = True


class OffloadLoad(_Model):
    key = "offload-load"
    assumptions = ("the load stream and the forward stream are otherwise unordered",)
    not_covered = ("eviction of the host copy during the load",)
    B = ("gpu", 0)

    def enabled(self):
        s, B, acts = self.s, self.B, []
        if not s.get("issued"):
            return [self.act("prefix hit: alloc block, issue host->GPU load", {B, "ld", "r"}, lambda m: m._issue())]
        ld = self.ledger.ops["ld"]
        if ld.state == "outstanding" and not s.get("landed"):
            acts.append(self.act("load stream copies", {B, "ld"}, lambda m: m._land()))
        if ld.state == "outstanding" and s.get("landed"):
            acts.append(self.act("load completes (event)", {B, "ld", "r"}, lambda m: m._complete()))
        fwd_ok = ld.state == "completed" if self.variant == "fixed" else True
        if fwd_ok and not s.get("fwd"):
            acts.append(self.act("forward reads the block", {B, "r"}, lambda m: m._forward()))
        return acts

    def done(self):
        return bool(self.s.get("fwd"))

    def _issue(self):
        self.h["b"] = self.ledger.alloc(self.B, "r")
        self.ledger.submit("ld", "load", "load-stream", dst=self.h["b"], payload=("r", self.h["b"].gen, "prefix"))
        self.s["issued"] = True
        if self.variant == "buggy":
            self.ledger.regions[self.B].ready = True     # marked usable at issue

    def _land(self):
        self.ledger.land("ld")
        self.s["landed"] = True

    def _complete(self):
        self.ledger.complete("ld", self.h["b"])

    def _forward(self):
        self.ledger.consume(self.h["b"], "r")
        self.s["fwd"] = True


MODELS = {m.key: m for m in (PDAbort, PDLease, PDNotify, OffloadLoad)}


def make(name: str):
    """'pd-abort:buggy' -> a factory of fresh model instances."""
    key, _, variant = name.partition(":")
    cls = MODELS[key]
    return lambda: cls(variant or "buggy")
