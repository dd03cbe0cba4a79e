"""The recording and delay hooks a real (threaded) implementation calls, for the model-free search.

A Probe is a thread-safe `EventSink` (the same event lines the engine writes, plus the calling thread's name) with
asynchronous operations (submit, land, complete, stop as separate events, from any thread) and checkpoints: points
where the calling thread could legally be slow (before a transfer is issued, before a completion is handled). A
checkpoint is a no-op unless the search installed a hold for it: then the thread waits there until the hold's
condition holds on the events recorded so far (or a bounded time passes), which reorders the run the way a stalled
thread, a preempted process or a late message would. Nothing is fabricated: a held thread later does exactly what it
would have done.

Reference: src/sdcguard/lifetime/realsearch.py:1-20 (code instrumented with a Probe: recording calls and
checkpoints, the points where work could legally be delayed).
"""
from __future__ import annotations

import threading
import time
from typing import Callable, Optional

from .adapter import EventSink

HOLD_LIMIT_S = 0.25          # a hold never blocks longer than this: the run goes on and is judged as it is


class Hold:
    """Hold the `occurrence`-th arrival of `thread` at checkpoint `name` until `until(events, start)` is true
    (start: the index of the first event recorded after the hold began)."""

    def __init__(self, thread: str, name: str, occurrence: int, until: Callable[[list, int], bool], text: str):
        self.thread, self.name, self.occurrence, self.until, self.text = thread, name, occurrence, until, text
        self.fired = False
        self.satisfied = False


class Probe(EventSink):
    def __init__(self, hold: Optional[Hold] = None):
        super().__init__()
        self.cv = threading.Condition()
        self.hold = hold
        self.checkpoints: list[dict] = []        # {"thread", "name", "occurrence", "at": index of the next event}
        self._seen: dict = {}

    def _emit(self, ev: dict) -> None:
        with self.cv:
            ev = {**ev, "thread": threading.current_thread().name}
            super()._emit(ev)
            self.cv.notify_all()

    # the recording calls of EventSink, made atomic (the generation table and the event order change together)
    def alloc(self, pool, idx, owner):
        with self.cv:
            super().alloc(pool, idx, owner)

    def free(self, pool, idx):
        with self.cv:
            super().free(pool, idx)

    def share(self, pool, idx, request):
        with self.cv:
            super().share(pool, idx, request)

    def local_write(self, pool, idx, by):
        with self.cv:
            super().local_write(pool, idx, by)

    def consume(self, pool, idx, request):
        with self.cv:
            super().consume(pool, idx, request)

    # asynchronous operations (the synchronous `transfer` of EventSink is submit + land + complete at once)
    def submit(self, kind: str, by: str, src: Optional[tuple], dst: Optional[tuple], src_gen=None, dst_gen=None) -> str:
        with self.cv:
            self._ops += 1
            op = f"{kind}{self._ops}"
            s = self.handle(*src) if src else None
            d = self.handle(*dst) if dst else None
            if s is not None and src_gen is not None:
                s[1] = src_gen
            if d is not None and dst_gen is not None:
                d[1] = dst_gen
            self._emit({"ev": "submit", "op": op, "kind": kind, "by": by, "src": s, "dst": d})
            return op

    def land(self, op: str) -> None:
        self._emit({"ev": "land", "op": op})

    def complete(self, op: str, mark: Optional[list] = None) -> None:
        self._emit({"ev": "complete", "op": op, "mark": mark})

    def stop(self, op: str) -> None:
        self._emit({"ev": "stop", "op": op})

    def handle_now(self, pool: str, idx: int) -> list:
        with self.cv:
            return self.handle(pool, idx)

    def checkpoint(self, name: str) -> None:
        me = threading.current_thread().name
        with self.cv:
            k = (me, name)
            n = self._seen.get(k, 0)
            self._seen[k] = n + 1
            self.checkpoints.append({"thread": me, "name": name, "occurrence": n, "at": len(self.events)})
            h = self.hold
            if h is None or h.fired or h.thread != me or h.name != name or h.occurrence != n:
                return
            h.fired = True
            start = len(self.events)
            deadline = time.monotonic() + HOLD_LIMIT_S
            while not h.until(self.events, start):
                left = deadline - time.monotonic()
                if left <= 0:
                    return
                self.cv.wait(left)
            h.satisfied = True
