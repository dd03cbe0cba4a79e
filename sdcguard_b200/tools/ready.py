"""Is this server's math being checked right now? Asked from outside, from its metrics.

    sdcguard ready http://127.0.0.1:8000 [--url http://127.0.0.1:8001 ...] [--probe] [--window 2] [--max-z 6]
    sdcguard ready --port 9400 --workers 2 [--host 127.0.0.1] [--probe URL]     # the vLLM plugin's exporters
        [--layers N] [--min-weights 0.5] [--gpus UUID,UUID] [--qualified decision.json] [--max-age-days D]
        [--strict-conditions] [--strict-alerts] [--json]

Reads every worker's /metrics twice, --window seconds apart (with --probe: two short requests to each worker in
between), and answers PROTECTED only if, on every worker:

  - its metrics are there, with checks on (sdcguard_protected 1);
  - linear layers are checked, every checked op has run, and every worker checks the same number of layers (at
    least --layers, and a share of the linear-layer weights of at least --min-weights, when given);
  - the alarm line is at most --max-z (a server told to alarm at z = 1000 never alarms);
  - check results have been read back at least once;
  - each worker is on its own GPU (with --gpus: exactly the GPUs given), and none restarted between the reads;
  - its checks went up between the reads while it produced tokens (its own token counter tells an idle worker from
    one whose checks stopped). A worker that produced no tokens leaves the answer IDLE: everything else holds but
    nothing shows the checks would run for the next request; --probe turns IDLE into a definite answer.

FAULT FOUND, whatever else holds: a worker counts a confirmed alert (an alert whose own evidence shows a wrong
result: a float64 recheck outside the rounding envelope, a replay that differed, a changed weight;
sdcguard_confirmed_alerts_total, or the alarm counter on a server that does not publish it). Unconfirmed alerts are
notes; --strict-alerts makes any alert FAULT FOUND.

With --qualified DECISION.json (written by `sdcguard decide` or `sdcguard qualify`): NOT QUALIFIED when the decision
was not ACCEPT; NOT THE QUALIFIED STACK when a worker's stack record differs from the one the decision was made on;
INCONCLUSIVE when either side records no stack or the decision is older than --max-age-days (or its policy's
ready.max_age_days; the smaller applies). The checks are held to what the qualification ran with: the weight share
at least the larger of --min-weights and the decision's arithmetic.min_weights_checked, the alarm line at most the
smaller of --max-z and the qualification's line, and every replay or scan the qualification had on still on; a
weaker setting is NOT PROTECTED, listing what is weaker. Where the server has gone beyond what the qualification
exercised (a longer prompt than any it sent), a note; INCONCLUSIVE with --strict-conditions.

Exit codes: 0 PROTECTED or IDLE, 1 FAULT FOUND, NOT PROTECTED, NOT THE QUALIFIED STACK or NOT QUALIFIED,
2 INCONCLUSIVE. For a readiness probe, any nonzero code keeps traffic away.

Reference: src/sdcguard/ready.py:1-80 (the conditions, verdict words and exit codes), `judge` :400, `qualified`
:245, `_weaker` :207.
"""
from __future__ import annotations

import argparse
import json
import time
from typing import Callable, Optional

from . import _client

DETECTORS = ("norms", "rope", "attn", "act", "spot", "weight_scan")


def _labels(m: dict, name: str) -> dict:
    rows = m.get(name + "{}") or []
    return dict(rows[0][0]) if rows else {}


def _stack(m: dict) -> dict:
    return _labels(m, "sdcguard_stack_info")


def _worker(m: dict) -> dict:
    return _labels(m, "sdcguard_worker_info")


def _confirmed(m: dict) -> float:
    if "sdcguard_confirmed_alerts_total" in m:
        return m["sdcguard_confirmed_alerts_total"]
    return m.get("sdcguard_alarms_total", 0)


def judge(first: list, second: list, max_z: float = 6.0, layers: Optional[int] = None,
          min_weights: Optional[float] = None, gpus: Optional[list] = None, strict_alerts: bool = False) -> dict:
    """The verdict from two reads of every worker's metrics (a pure function of the metrics)."""
    if isinstance(first, dict) or first is None:          # one worker given bare
        first, second = [first], [second]
    notes = []
    missing = [i for i, (a, b) in enumerate(zip(first, second)) if a is None or b is None]
    if missing:
        return {"verdict": "NOT PROTECTED", "why": [f"worker {i}: no metrics (server down, or not this library's "
                                                     "server)" for i in missing], "notes": notes}
    faults = []
    for i, m in enumerate(second):
        c = _confirmed(m)
        if c > 0:
            faults.append(f"worker {i}: {c:g} confirmed alerts")
        elif m.get("sdcguard_alerts_total", 0) > 0:
            (faults if strict_alerts else notes).append(
                f"worker {i}: {m['sdcguard_alerts_total']:g} alerts not confirmed by their own evidence")
    if faults:
        return {"verdict": "FAULT FOUND", "why": faults, "notes": notes}
    restarted = [i for i, (a, b) in enumerate(zip(first, second))
                 if (_worker(a).get("started"), _worker(a).get("pid")) != (_worker(b).get("started"),
                                                                             _worker(b).get("pid"))]
    if restarted:
        return {"verdict": "INCONCLUSIVE", "why": [f"worker {i} restarted between the reads" for i in restarted],
                "notes": notes}
    why = []
    for i, m in enumerate(second):
        if m.get("sdcguard_protected", 0) != 1:
            why.append(f"worker {i}: checks are off (sdcguard_protected 0)")
            continue
        if m.get("sdcguard_alarm_line", 1e9) > max_z:
            why.append(f"worker {i}: alarm line {m.get('sdcguard_alarm_line')} above {max_z:g}")
        ops, checked = m.get("sdcguard_ops_total", 0), m.get("sdcguard_ops_checked", 0)
        if ops and checked < ops and m.get("sdcguard_polls_total", 0) >= 1:
            why.append(f"worker {i}: {ops - checked:g} of {ops:g} checked ops never ran")
        lc = m.get("sdcguard_layers_checked")
        if lc is not None and lc <= 0:
            why.append(f"worker {i}: no linear layer is checked")
        if layers is not None and (lc or 0) < layers:
            why.append(f"worker {i}: {lc or 0:g} layers checked, {layers} required")
        ratio = m.get("sdcguard_weights_checked_ratio")
        if min_weights is not None and (ratio if ratio is not None else 0.0) < min_weights:
            why.append(f"worker {i}: {ratio or 0:.0%} of the linear-layer weights checked, {min_weights:.0%} "
                       "required")
    counts = {m.get("sdcguard_layers_checked") for m in second}
    if len(counts) > 1:
        why.append(f"the workers check different numbers of layers ({sorted(c for c in counts if c is not None)})")
    uuids = [_worker(m).get("uuid") for m in second]
    if len(set(uuids)) != len(uuids):
        why.append("two workers report the same GPU")
    if gpus is not None and sorted(uuids) != sorted(gpus):
        why.append(f"the workers run on {sorted(uuids)}, not the GPUs given ({sorted(gpus)})")
    if why:
        return {"verdict": "NOT PROTECTED", "why": why, "notes": notes}
    if any(m.get("sdcguard_polls_total", 0) < 1 for m in second):
        return {"verdict": "INCONCLUSIVE", "why": ["no check result has been read back yet on a worker (send a "
                                                   "request, or use --probe)"], "notes": notes}
    idle, moved = [], []
    for i, (a, b) in enumerate(zip(first, second)):
        tokens = b.get("sdcguard_generated_tokens_total", 0) - a.get("sdcguard_generated_tokens_total", 0)
        checks = b.get("sdcguard_checks_total", 0) - a.get("sdcguard_checks_total", 0)
        if tokens > 0 and checks <= 0:
            why.append(f"worker {i}: produced {tokens:g} tokens while its checks did not move")
        elif tokens <= 0:
            idle.append(i)
        else:
            moved.append((checks, tokens))
    if why:
        return {"verdict": "NOT PROTECTED", "why": why, "notes": notes}
    if idle:
        return {"verdict": "IDLE", "why": [f"worker {i}: no tokens between the reads" for i in idle], "notes": notes}
    return {"verdict": "PROTECTED", "why": [], "notes": notes, "checks_between_reads": sum(c for c, _ in moved),
            "tokens_between_reads": sum(t for _, t in moved)}


def _truthy(v) -> bool:
    return str(v).lower() in ("1", "true", "on", "yes")


def weaker(then: dict, now: dict) -> list:
    """Check settings of now that are weaker than the qualification's (then): a smaller share, a higher alarm line,
    a replay or scan switched off."""
    out = []
    try:
        if float(now.get("share", 1)) < float(then.get("share", 1)) - 1e-9:
            out.append(f"share {now.get('share')} < {then.get('share')} qualified")
        if float(now.get("z", 0)) > float(then.get("z", 1e9)) + 1e-9:
            out.append(f"alarm line {now.get('z')} > {then.get('z')} qualified")
    except (TypeError, ValueError):
        out.append("unreadable share or alarm line")
    for d in DETECTORS:
        if _truthy(then.get(d)) and not _truthy(now.get(d)):
            out.append(f"{d} check off (on when qualified)")
    return out


def qualified(second: list, decision: dict, max_age_days: Optional[float] = None, min_weights: Optional[float] = None,
              max_z: float = 6.0, strict_conditions: bool = False, now: Optional[float] = None) -> Optional[dict]:
    """The qualification verdict, or None when every worker serves the qualified stack under checks as strong."""
    from .decide import still_applies
    if isinstance(second, dict):
        second = [second]
    if decision.get("decision") != "ACCEPT":
        return {"verdict": "NOT QUALIFIED", "why": [f"the decision was {decision.get('decision')}"]}
    pol_age = ((decision.get("policy") or {}).get("ready") or {}).get("max_age_days")
    ages = [a for a in (max_age_days, pol_age) if a is not None]
    created = decision.get("created_unix")
    if ages:
        if created is None:
            return {"verdict": "INCONCLUSIVE", "why": ["the decision records no creation time"]}
        age = ((now or time.time()) - created) / 86400.0
        if age > min(ages):
            return {"verdict": "INCONCLUSIVE", "why": [f"the decision is {age:.1f} days old (limit {min(ages):g})"]}
    why, unsure, notes = [], [], []
    for i, m in enumerate(second):
        stack = _stack(m)
        stack.setdefault("gpu", _worker(m).get("uuid"))
        r = still_applies(decision, stack or None)
        if r["applies"] is None:
            unsure.append(f"worker {i}: {r['why']}")
        elif not r["applies"]:
            why += [f"worker {i}: {d}" for d in r["differences"]]
    if why:
        return {"verdict": "NOT THE QUALIFIED STACK", "why": why}
    if unsure:
        return {"verdict": "INCONCLUSIVE", "why": unsure}
    then = (decision.get("scope") or {}).get("settings") or {}
    pol_w = ((decision.get("policy") or {}).get("arithmetic") or {}).get("min_weights_checked")
    need_w = max([w for w in (min_weights, pol_w) if w is not None], default=None)
    weak = []
    for i, m in enumerate(second):
        now_s = _labels(m, "sdcguard_protection_info")
        if then:
            weak += [f"worker {i}: {w}" for w in weaker(then, now_s)]
        ratio = m.get("sdcguard_weights_checked_ratio")
        if need_w is not None and (ratio if ratio is not None else 0.0) < need_w:
            weak.append(f"worker {i}: {ratio or 0:.0%} of the weights checked, the qualification needs {need_w:.0%}")
        try:
            if then and float(now_s.get("z", max_z)) > min(max_z, float(then.get("z", max_z))):
                weak.append(f"worker {i}: alarm line {now_s.get('z')} above the qualified {then.get('z')}")
        except ValueError:
            weak.append(f"worker {i}: unreadable alarm line")
    if not then:
        notes.append("the decision records no check settings: only the command line's requirements apply")
    if weak:
        return {"verdict": "NOT PROTECTED", "why": sorted(set(weak)), "notes": notes}
    tested = (decision.get("tested") or {}).get("longest_prompt")
    longest = max((m.get("sdcguard_longest_prompt_tokens", 0) for m in second), default=0)
    if tested is not None and longest > tested:
        msg = f"the server served a {longest:g}-token prompt, longer than any the qualification sent ({tested})"
        if strict_conditions:
            return {"verdict": "INCONCLUSIVE", "why": [msg]}
        notes.append(msg)
    return {"verdict": None, "notes": notes}


def check(urls, probe: bool = False, window: float = 2.0, max_z: float = 6.0, layers: Optional[int] = None,
          min_weights: Optional[float] = None, gpus: Optional[list] = None, decision: Optional[dict] = None,
          max_age_days: Optional[float] = None, strict_conditions: bool = False, strict_alerts: bool = False,
          scrape: Callable = _client.scrape, complete: Callable = _client.complete, wait: Optional[float] = None,
          probe_url: Optional[str] = None) -> dict:
    urls = [urls] if isinstance(urls, str) else list(urls)
    window = wait if wait is not None else window
    first = [scrape(u) for u in urls]
    t0 = time.time()
    if probe:
        # the server's API (one for all workers), or each worker's own URL (this package's HTTP server)
        targets = [probe_url] if probe_url else [u for u, m in zip(urls, first) if m is not None]
        for u in targets:
            for i in range(2):
                try:
                    complete(u, [1 + i, 2, 3, 4], 4)
                except Exception:  # noqa: BLE001  (a failed probe shows as checks that did not move)
                    pass
    left = window - (time.time() - t0)
    if left > 0 and not probe:
        time.sleep(left)
    second = [scrape(u) for u in urls]
    r = judge(first, second, max_z, layers, min_weights, gpus, strict_alerts)
    if decision is not None and r["verdict"] in ("PROTECTED", "IDLE") and None not in second:
        q = qualified(second, decision, max_age_days, min_weights, max_z, strict_conditions)
        if q is not None and q.get("verdict"):
            r = dict(q, notes=r.get("notes", []) + q.get("notes", []))
        elif q is not None:
            r["notes"] = r.get("notes", []) + q.get("notes", [])
    r["workers"] = [{"url": u, "stack": _stack(m or {}), "worker": _worker(m or {})} for u, m in zip(urls, second)]
    r["stack"] = r["workers"][0]["stack"] if r["workers"] else {}
    return r


EXIT = {"PROTECTED": 0, "IDLE": 0, "INCONCLUSIVE": 2}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="sdcguard ready", description=__doc__.split("\n\n")[0])
    ap.add_argument("url", nargs="?")
    ap.add_argument("--url", dest="urls", action="append", default=[], help="another worker (repeat)")
    ap.add_argument("--port", type=int, help="first worker's metrics port (SDCGUARD_METRICS_PORT of a vLLM server "
                                            "with this package's plugin; worker i answers on port + i)")
    ap.add_argument("--workers", type=int, default=1)
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--probe", nargs="?", const=True, default=False, metavar="API_URL",
                    help="send two short requests between the reads (to the worker URLs, or to API_URL when the "
                         "metrics come from exporters)")
    ap.add_argument("--window", "--wait", type=float, default=2.0)
    ap.add_argument("--max-z", type=float, default=6.0)
    ap.add_argument("--layers", type=int)
    ap.add_argument("--min-weights", type=float)
    ap.add_argument("--gpus", help="the GPUs the workers must run on (UUIDs, comma-separated)")
    ap.add_argument("--qualified", metavar="DECISION")
    ap.add_argument("--max-age-days", type=float)
    ap.add_argument("--strict-conditions", action="store_true")
    ap.add_argument("--strict-alerts", action="store_true")
    ap.add_argument("--json", action="store_true")
    a = ap.parse_args(argv)
    urls = ([a.url] if a.url else []) + a.urls
    if a.port is not None:
        urls += [f"http://{a.host}:{a.port + i}" for i in range(max(1, a.workers))]
    if not urls:
        ap.error("give at least one worker URL (or --port)")
    dec = None
    if a.qualified:
        with open(a.qualified) as f:
            dec = json.load(f)
    probe_to = a.probe if isinstance(a.probe, str) else None
    r = check(urls, bool(a.probe), a.window, a.max_z, a.layers, a.min_weights,
              [g.strip() for g in a.gpus.split(",")] if a.gpus else None, dec, a.max_age_days,
              a.strict_conditions, a.strict_alerts, probe_url=probe_to)
    if a.json:
        print(json.dumps(r, indent=1))
    else:
        print(r["verdict"])
        for w in r.get("why") or []:
            print(f"  {w}")
        for n in r.get("notes") or []:
            print(f"  note: {n}")
    return EXIT.get(r["verdict"], 1)


if __name__ == "__main__":
    raise SystemExit(main())
