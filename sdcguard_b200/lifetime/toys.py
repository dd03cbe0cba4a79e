"""Small real implementations of KV-transfer protocols, for demonstrating and testing the model-free search
(`realsearch.search`). They are real code, not models: threads, real timers and queues, and a byte store the
transfers really copy. Each records through a `Probe` and marks the points where a thread could legally be slow
with `probe.checkpoint(...)`. The search is given only `make()` and `run()`; it is not told where the bug is.

ToyPush    the prefill side writes KV into a block the decode side allocated; the decode side times out a slow
           request and moves on to the next one. fixed=True: on timeout the decode side asks the prefill side to
           stop and frees the block only after it answers that no write is outstanding.
ToyPull    the decode side pulls KV from a block the prefill side holds under a lease that expires on a timer.
           fixed=True: the consumer pins the lease before reading; a pin after expiry fails the request (allowed).
ToyWakeup  a lost wakeup (liveness): a completion that lands between the waiter's "done?" test and its wait is
           missed. fixed=True: test and wait under one lock.

run() returns {"finished": bool, "outcomes": {...}}: finished is False when a thread did not end by the deadline.

Reference: src/sdcguard/lifetime/toys.py:1-20 (ToyPull, ToyPush, ToyWakeup and what each fixed variant changes).
"""
from __future__ import annotations

import queue
import threading
import time

from .probe import Probe

TIMEOUT_S = 0.05          # decode-side request timeout / lease length
DEADLINE_S = 1.0          # a run that has not finished by then is a liveness finding


def _join(threads, deadline: float) -> bool:
    end = time.monotonic() + deadline
    for t in threads:
        t.join(max(0.0, end - time.monotonic()))
    return not any(t.is_alive() for t in threads)


class ToyPush:
    def __init__(self, fixed: bool = False):
        self.fixed = fixed
        self.store = {0: b""}                       # one decode block: block 0
        self.to_prefill: queue.Queue = queue.Queue()
        self.to_decode: queue.Queue = queue.Queue()
        self.outcomes: dict = {}

    def prefill(self, p: Probe) -> None:
        while True:
            msg = self.to_prefill.get()
            if msg is None:
                return
            if msg[0] == "stop":                    # fixed protocol: answer once nothing is outstanding
                self.to_decode.put(("stopped", msg[1]))
                continue
            _, req, block, gen = msg
            p.checkpoint("prefill.before_write")
            op = p.submit("write", "prefill", None, ("decode", block), dst_gen=gen)
            self.store[block] = f"kv-of-{req}".encode()
            p.land(op)
            p.complete(op, [["decode", block], gen])
            self.to_decode.put(("done", req, op))

    def decode(self, p: Probe) -> None:
        for req in ("r1", "r2"):
            p.alloc("decode", 0, req)
            gen = p.handle_now("decode", 0)[1]
            self.to_prefill.put(("write", req, 0, gen))
            try:
                while True:
                    msg = self.to_decode.get(timeout=TIMEOUT_S if req == "r1" else DEADLINE_S / 2)
                    if msg[0] == "done" and msg[1] == req:
                        break
            except queue.Empty:
                self.outcomes[req] = "timed_out"
                if self.fixed:
                    self.to_prefill.put(("stop", req))
                    while True:                     # drain: the write (if issued) finishes before the answer
                        m = self.to_decode.get(timeout=DEADLINE_S / 2)
                        if m[0] == "stopped":
                            break
                p.free("decode", 0)
                continue
            p.consume("decode", 0, req)
            self.outcomes[req] = "served"
            p.free("decode", 0)
        self.to_prefill.put(None)

    def run(self, p: Probe) -> dict:
        ts = [threading.Thread(target=self.prefill, args=(p,), name="prefill", daemon=True),
              threading.Thread(target=self.decode, args=(p,), name="decode", daemon=True)]
        for t in ts:
            t.start()
        return {"finished": _join(ts, DEADLINE_S), "outcomes": dict(self.outcomes)}


class ToyPull:
    def __init__(self, fixed: bool = False):
        self.fixed = fixed
        self.store = {0: b""}
        self.lock = threading.Lock()
        self.pinned: set = set()             # requests whose lease is pinned
        self.expired: set = set()            # requests whose lease expired
        self.to_decode: queue.Queue = queue.Queue()
        self.outcomes: dict = {}

    def prefill(self, p: Probe) -> None:
        for req in ("r1", "r2"):
            p.alloc("prefill", 0, req)
            p.local_write("prefill", 0, req)
            self.store[0] = f"kv-of-{req}".encode()
            gen = p.handle_now("prefill", 0)[1]
            self.to_decode.put((req, 0, gen))
            if req == "r2":
                return
            time.sleep(TIMEOUT_S)                   # the lease
            p.checkpoint("prefill.lease_expiry")
            while True:
                with self.lock:
                    if req not in self.pinned:
                        self.expired.add(req)
                        break
                time.sleep(0.001)                   # a pinned lease does not expire: wait for the unpin
            p.free("prefill", 0)

    def decode(self, p: Probe) -> None:
        for _ in range(2):
            req, block, gen = self.to_decode.get(timeout=DEADLINE_S / 2)
            p.checkpoint("decode.before_read")
            if self.fixed:
                with self.lock:
                    if req in self.expired:
                        self.outcomes[req] = "failed_lease_expired"
                        continue
                    self.pinned.add(req)
            p.alloc("decode", 1, req)
            op = p.submit("read", "decode", ("prefill", block), ("decode", 1), src_gen=gen)
            data = self.store[block]
            p.land(op)
            p.complete(op, p.handle_now("decode", 1))
            if self.fixed:
                with self.lock:
                    self.pinned.discard(req)
            p.consume("decode", 1, req)
            self.outcomes[req] = "served" if data == f"kv-of-{req}".encode() else "served_wrong_data"
            p.free("decode", 1)

    def run(self, p: Probe) -> dict:
        ts = [threading.Thread(target=self.prefill, args=(p,), name="prefill", daemon=True),
              threading.Thread(target=self.decode, args=(p,), name="decode", daemon=True)]
        for t in ts:
            t.start()
        return {"finished": _join(ts, DEADLINE_S), "outcomes": dict(self.outcomes)}


class ToyWakeup:
    def __init__(self, fixed: bool = False):
        self.fixed = fixed
        self.done = False
        self.cv = threading.Condition()
        self.outcomes: dict = {}

    def worker(self, p: Probe) -> None:
        p.alloc("decode", 0, "r1")
        op = p.submit("write", "worker", None, ("decode", 0))
        p.land(op)
        p.checkpoint("worker.before_signal")
        with self.cv:
            self.done = True
            self.cv.notify_all()
        p.complete(op, p.handle_now("decode", 0))

    def waiter(self, p: Probe) -> None:
        if self.fixed:
            with self.cv:
                self.cv.wait_for(lambda: self.done, timeout=DEADLINE_S * 2)
        else:
            d = self.done                           # test ...
            p.checkpoint("waiter.between_test_and_wait")
            if not d:
                with self.cv:                       # ... then wait: a signal in between is lost
                    self.cv.wait(timeout=DEADLINE_S * 2)
        self.outcomes["r1"] = "woken" if self.done else "timed_out"

    def run(self, p: Probe) -> dict:
        ts = [threading.Thread(target=self.waiter, args=(p,), name="waiter", daemon=True),
              threading.Thread(target=self.worker, args=(p,), name="worker", daemon=True)]
        for t in ts:
            t.start()
        return {"finished": _join(ts, DEADLINE_S), "outcomes": dict(self.outcomes)}


TOYS = {"push": ToyPush, "pull": ToyPull, "wakeup": ToyWakeup}
