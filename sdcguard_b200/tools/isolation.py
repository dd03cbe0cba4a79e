"""Does one request's answer depend on other requests? Two probes against a running server of this package
(`sdcguard serve`, or any server with the same token-id completions API):

    python -m sdcguard_b200.tools.isolation http://127.0.0.1:8000 --probes 4 --primers 3 --repeats 2

A server can compute every GEMM right and still answer one request with another's data: a stale buffer, a KV page
reused too early, a cached prefix read from the wrong pages. Checks of the arithmetic cannot see these.

1. Primer dependence. A probe prompt is sent alone, greedy, right after a primer request that also ran alone; each
   (primer, probe) pair is repeated. On an isolated server the probe's tokens do not depend on which primer came
   before. The control is the probe after the same primer, repeated: it must agree exactly, otherwise the server is
   not deterministic at batch size 1 and the probe can judge nothing.
2. Concurrency. The probe is sent while other requests of different prompts and lengths run in the same batches; a
   batch-dependent answer is reported.
3. Cancellation under shared prefixes. Groups of requests share a long prompt head (a server with a prefix cache
   shares its blocks) and differ in a short tail. Each is answered alone twice (the control), then all are sent at
   once together with more requests of the same heads that are streamed and dropped after their first event, so
   the server ends them mid-flight and hands their KV pages back while the others still read theirs. Every answer
   under that load must equal its solo answer. (The reference's canary probe asks a trained model to repeat a code
   from its context and looks for another request's code; random-init weights copy nothing, so here the solo
   answer is the witness.)

Verdicts: LEAK (a probe's answer changed with the primer in the same way every time that primer came before it,
while every control repeat agreed; or a concurrent answer differed from the solo one on a server whose solo repeats
agree), NO LEAK SEEN (neither, with every control agreeing), INCONCLUSIVE (a control disagreed, a request failed, or
answers changed in ways that do not repeat with their primer: one differing token cannot be told from a server that
is not deterministic). NO LEAK SEEN covers these prompts, this load and this server only. Exit 0 / 1 (LEAK) / 2.

Reference: src/sdcguard/isolation.py:1-40 (the probes and verdict rules), :179 (the canary probe: shared document
prefixes, concurrent requests, a share of them cancelled after their first chunk).
"""
from __future__ import annotations

import argparse
import json
import random
import threading
from typing import Callable, Optional

from . import _client

SCHEMA = "sdcguard.isolation/1"


def _first_diff(a, b) -> Optional[int]:
    if a is None or b is None:
        return 0
    for i, (x, y) in enumerate(zip(a, b)):
        if x != y:
            return i
    return None if len(a) == len(b) else min(len(a), len(b))


def primer_probe(base: str, probe: list, primers: list, repeats: int, tokens: int, complete: Callable) -> dict:
    """The probe's answers after each primer, `repeats` times each (primer and probe sent one after the other)."""
    answers: dict = {}
    for rep in range(repeats):
        for pi, pr in enumerate(primers):
            complete(base, pr, tokens)
            answers.setdefault(pi, []).append(complete(base, probe, tokens))
    controls_agree = all(all(a == ans[0] for a in ans) for ans in answers.values())
    # the answer after each primer (its repeats agree), and whether it differs from the first primer's
    per = {pi: ans[0] for pi, ans in answers.items() if all(a == ans[0] for a in ans)}
    base_ans = per.get(0)
    changed_repeatably = [pi for pi, a in per.items() if pi != 0 and base_ans is not None and a != base_ans]
    unstable = [pi for pi, ans in answers.items() if pi not in per]
    if not controls_agree:
        verdict = "INCONCLUSIVE"
    elif changed_repeatably:
        verdict = "LEAK"
    else:
        verdict = "NO LEAK SEEN"
    return {"verdict": verdict, "controls_agree": controls_agree, "unstable_primers": unstable,
            "primers_changing_the_answer": changed_repeatably,
            "first_difference": {pi: _first_diff(base_ans, per[pi]) for pi in changed_repeatably}}


def concurrency_probe(base: str, probe: list, others: list, tokens: int, complete: Callable) -> dict:
    solo = complete(base, probe, tokens)
    again = complete(base, probe, tokens)
    got: dict = {}

    def fire(key, ids):
        try:
            got[key] = complete(base, ids, tokens)
        except Exception as e:  # noqa: BLE001  (a failed request makes the probe inconclusive)
            got[key] = e
    th = [threading.Thread(target=fire, args=(i, x)) for i, x in enumerate(others)]
    th.append(threading.Thread(target=fire, args=("probe", probe)))
    for t in th:
        t.start()
    for t in th:
        t.join()
    mixed = got.get("probe")
    failed = any(isinstance(v, Exception) for v in got.values())
    if failed or solo != again:
        verdict = "INCONCLUSIVE"
    else:
        verdict = "LEAK" if mixed != solo else "NO LEAK SEEN"
    return {"verdict": verdict, "solo_repeats_agree": solo == again, "failed_requests": failed,
            "first_difference": None if isinstance(mixed, Exception) else _first_diff(solo, mixed)}


def cancel_probe(base: str, groups: int = 4, per_group: int = 4, head: int = 96, tail: int = 8, tokens: int = 16,
                 cancels_per_group: int = 2, seed: int = 0, vocab: int = 1000, complete: Callable = _client.complete,
                 cancel: Callable = _client.stream_cancel) -> dict:
    """Probe 3 of the module docstring. `cancel(base, ids, n)` starts a streamed request and drops it after its
    first event."""
    rng = random.Random(seed * 104729 + 3)
    heads = [[rng.randrange(vocab) for _ in range(head)] for _ in range(groups)]
    reqs = [{"group": g, "ids": heads[g] + [rng.randrange(vocab) for _ in range(tail)]}
            for g in range(groups) for _ in range(per_group)]
    drops = [{"group": g, "ids": heads[g] + [rng.randrange(vocab) for _ in range(tail)]}
             for g in range(groups) for _ in range(cancels_per_group)]
    try:
        solo = [complete(base, r["ids"], tokens) for r in reqs]
        again = [complete(base, r["ids"], tokens) for r in reqs]
    except Exception as e:  # noqa: BLE001
        return {"verdict": "INCONCLUSIVE", "error": f"solo request failed: {str(e)[:300]}"}
    controls = [i for i, (a, b) in enumerate(zip(solo, again)) if a != b]
    got: dict = {}
    errors: list = []

    def answer(i):
        try:
            got[i] = complete(base, reqs[i]["ids"], tokens)
        except Exception as e:  # noqa: BLE001
            errors.append(f"request {i}: {str(e)[:200]}")

    dropped: list = []

    def drop(j):
        try:
            if cancel(base, drops[j]["ids"], 4 * tokens):
                dropped.append(j)
        except Exception as e:  # noqa: BLE001  (a stream that could not start was not dropped mid-flight)
            errors.append(f"cancelled request {j}: {str(e)[:200]}")
    th = [threading.Thread(target=drop, args=(j,)) for j in range(len(drops))]
    th += [threading.Thread(target=answer, args=(i,)) for i in range(len(reqs))]
    for t in th:
        t.start()
    for t in th:
        t.join()
    changed = [{"request": i, "group": reqs[i]["group"], "first_difference": _first_diff(solo[i], got[i])}
               for i in range(len(reqs)) if i in got and got[i] != solo[i] and i not in controls]
    answered = sum(1 for i in range(len(reqs)) if i in got)
    if changed and not controls:
        verdict = "LEAK"
    elif controls or answered < len(reqs) or changed or not dropped:
        verdict = "INCONCLUSIVE"          # (no stream dropped mid-flight: the load this probe is for never ran)
    else:
        verdict = "NO LEAK SEEN"
    return {"verdict": verdict, "requests": len(reqs), "cancelled": len(drops), "dropped_mid_flight": len(dropped),
            "answered": answered,
            "controls_disagree": controls, "changed_under_load": changed, "errors": errors[:10]}


def run(base: str, probes: int = 4, primers: int = 3, repeats: int = 2, prompt: int = 24, tokens: int = 16,
        others: int = 8, seed: int = 0, vocab: int = 1000, complete: Callable = _client.complete,
        cancellation: bool = True, cancel: Callable = _client.stream_cancel) -> dict:
    rng = random.Random(seed)
    rows = []
    for p in range(probes):
        probe = [rng.randrange(vocab) for _ in range(prompt)]
        prim = [[rng.randrange(vocab) for _ in range(rng.randrange(8, 6 * prompt))] for _ in range(primers)]
        conc = [[rng.randrange(vocab) for _ in range(rng.randrange(8, 6 * prompt))] for _ in range(others)]
        try:
            a = primer_probe(base, probe, prim, repeats, tokens, complete)
            b = concurrency_probe(base, probe, conc, tokens, complete)
        except Exception as e:  # noqa: BLE001
            rows.append({"probe": p, "verdict": "INCONCLUSIVE", "error": str(e)[:300]})
            continue
        v = ("LEAK" if "LEAK" in (a["verdict"], b["verdict"]) else
             "INCONCLUSIVE" if "INCONCLUSIVE" in (a["verdict"], b["verdict"]) else "NO LEAK SEEN")
        rows.append({"probe": p, "verdict": v, "primer": a, "concurrency": b})
    cp = (cancel_probe(base, tokens=tokens, seed=seed, vocab=vocab, complete=complete, cancel=cancel)
          if cancellation else None)
    verdicts = [r["verdict"] for r in rows] + ([cp["verdict"]] if cp else [])
    verdict = ("LEAK" if "LEAK" in verdicts else "INCONCLUSIVE" if "INCONCLUSIVE" in verdicts or not rows
               else "NO LEAK SEEN")
    why = []
    for r in rows:
        if "error" in r:
            why.append(f"probe {r['probe']}: a request failed ({r['error'][:120]})")
            continue
        a, b = r["primer"], r["concurrency"]
        if a["primers_changing_the_answer"]:
            why.append(f"probe {r['probe']}: primers {a['primers_changing_the_answer']} changed its answer, the same "
                       "way on every repeat")
        if not a["controls_agree"]:
            why.append(f"probe {r['probe']}: repeats after the same primer disagree (the server is not "
                       "deterministic at batch size 1)")
        if b["verdict"] == "LEAK":
            why.append(f"probe {r['probe']}: its answer changed when other requests shared its batches (first "
                       f"difference at token {b['first_difference']})")
        elif b["verdict"] == "INCONCLUSIVE":
            why.append(f"probe {r['probe']}: the concurrency probe was inconclusive")
    if cp and cp["verdict"] == "LEAK":
        why.append(f"cancellation: {len(cp['changed_under_load'])} answers changed while requests of the same "
                   f"prompt heads were dropped mid-flight (their solo answers repeat exactly)")
    elif cp and cp["verdict"] == "INCONCLUSIVE":
        why.append("cancellation: " + (cp.get("error") or
                                       ("solo answers do not repeat" if cp["controls_disagree"] else
                                        "requests failed or answers changed beside solo answers that do not repeat")))
    differing = sum(len(r["primer"]["primers_changing_the_answer"]) for r in rows if "primer" in r)
    return {"schema": SCHEMA, "url": base, "verdict": verdict, "why": why, "probes": rows, "cancellation": cp,
            "primer": {"pairs": probes * (primers - 1), "pairs_differing": differing},
            "probe_set": {"probes": probes, "primers": primers, "repeats": repeats, "prompt": prompt,
                          "tokens": tokens, "others": others, "seed": seed},
            "scope": "these prompts, this load and this server only"}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="sdcguard isolation")
    ap.add_argument("url")
    ap.add_argument("--probes", type=int, default=4)
    ap.add_argument("--primers", type=int, default=3)
    ap.add_argument("--repeats", type=int, default=2)
    ap.add_argument("--tokens", type=int, default=16)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cancel", action="store_true", help="skip the cancellation probe")
    ap.add_argument("--out")
    a = ap.parse_args(argv)
    r = run(a.url, a.probes, a.primers, a.repeats, tokens=a.tokens, seed=a.seed, cancellation=not a.no_cancel)
    if a.out:
        with open(a.out, "w") as f:
            json.dump(r, f, indent=1)
    print(json.dumps({k: v for k, v in r.items() if k != "probes"}))
    return {"NO LEAK SEEN": 0, "LEAK": 1}.get(r["verdict"], 2)


if __name__ == "__main__":
    raise SystemExit(main())
