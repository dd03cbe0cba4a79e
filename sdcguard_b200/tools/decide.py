"""One decision on one proposed change to a serving stack (a library, driver or engine upgrade, fp8, a kernel or
parallelism setting), with its questions kept apart and each answered from its own evidence.

    sdcguard decide --out decision.json \\
        --policy policy.json                       # what the team accepts (below; every key optional)
        --quality check.json                       # `gate model-check` of the candidate against the trusted reference
        --gate verdicts.json                       # `gate compare`: the kept GEMM cases, before and after
        --kernels before.json after.json           # `sdcguard kernels parse` of each stack's cuBLASLt log
        --kernel-test tested.json                  # `sdcguard kernels test` of the candidate's inventory, on it
        --alerts alerts.jsonl                      # the candidate server's alert log (SDCGUARD_LOG)
        --plugin-metrics w0.txt [w1.txt ...]       # each worker's /metrics at the end of the candidate's run
        --perf before.json after.json              # `sdcguard perf` of each
        --isolation iso.json                       # `sdcguard isolation` of the candidate
        --consistency cons.json [base_cons.json]   # `sdcguard consistency` of the candidate (and of the baseline)
    sdcguard decide --applies decision.json --url http://127.0.0.1:8000   # does it still apply to that server?

Sections and their words:

1  arithmetic     FAULT / NO FAULT OBSERVED / INCONCLUSIVE. Judged against recomputation (float64, exact replays,
                  the spot check's rigorous bound), never against the old stack. Sources: the server's alerts (they
                  count as evidence of no fault only when every worker's metrics show checked layers, checks that
                  ran and results read back, a checked weight share of at least arithmetic.min_weights_checked, and
                  as many alert records as the workers counted), the kept GEMM cases of the upgrade gate (count when
                  one case was judged on both stacks) and the kernel test (counts when one call ran and was judged
                  on the workload's own kernel). A confirmed wrong output is a FAULT whatever else shows.
1a weights        CHANGED / VERIFIED / NO CHANGE SEEN / UNMEASURED: a weight-scan finding, a repair, or a recheck
                  that blames the weights is CHANGED; VERIFIED needs the scan to have compared every entry on every
                  worker; the ABFT checks alone see a changed weight only once it moves an output past the line.
1b quantization   WRONG / RIGHT / UNMEASURED: the fp8 layers' activation-quantization replays.
2  approximation  WITHIN / OUTSIDE / UNMEASURED: `gate model-check` (PASS, WARN with quality.accept_warn, the
                  policy's max_mean_kl and min_top1).
3  performance    MEETS / MISSES / UNMEASURED from `perf --compare` of the two runs: a required gain that does not
                  show past the noise, or a p99 limit passed (outside the noise), MISSES.
4  isolation      LEAK / NO LEAK SEEN / UNMEASURED.
4b consistency    CONSISTENT / INCONSISTENT / UNMEASURED, judged against the baseline's own decode/prefill gaps.
5  scope          the stacks, the kernels the change added and dropped, added kernels with a known issue or that no
                  test ran, what no source checks, and the candidate stack's fingerprint.

Every section states its effect: reject, missing (a needed answer is absent), ok or info. The decision is REJECT
when any section rejects (a FAULT, changed weights, WRONG quantization, OUTSIDE, a LEAK, INCONSISTENT, a required
performance target MISSES), otherwise NOT DECIDED when an answer is missing (arithmetic not NO FAULT OBSERVED,
approximation UNMEASURED, a required section UNMEASURED), otherwise ACCEPT: no reason to reject was found within
the scope listed. Exit 0 ACCEPT, 1 REJECT, 2 NOT DECIDED.

Policy (JSON; the reference's policy files are read unchanged):
    {"arithmetic": {"min_weights_checked": 0.5},
     "quality": {"accept_warn": false, "max_mean_kl": null, "min_top1": null},
     "performance": {"required": false, "min_throughput_gain": 0.0, "max_ttft_p99_increase": null,
                     "max_itl_p99_increase": null},
     "isolation": {"required": false}, "consistency": {"required": false}, "ready": {"max_age_days": null}}

Reference: src/sdcguard/decide.py:1-100 (sections, verdict words, decision rule and policy keys), `arithmetic` :274,
`weights_section` :378, `performance` :471, `scope` :581, `still_applies` :613.
"""
from __future__ import annotations

import argparse
import copy
import hashlib
import json
import os
import time
from dataclasses import dataclass, field
from typing import Optional

from . import _client

SCHEMA = "sdcguard.decision/1"
DEFAULT_POLICY = {"arithmetic": {"min_weights_checked": 0.5},
                  "quality": {"accept_warn": False, "max_mean_kl": None, "min_top1": None},
                  "performance": {"required": False, "min_throughput_gain": 0.0, "max_ttft_p99_increase": None,
                                  "max_itl_p99_increase": None},
                  "isolation": {"required": False},
                  "consistency": {"required": False},
                  "ready": {"max_age_days": None}}
NOT_CHECKED = ("kernels outside the checked GEMMs and replays (sampling, embedding, the library GEMMs of layers "
               "outside the checked share): only through the quality check",
               "requests unlike the quality check's prompts and the perf load",
               "faults that need the workload's own data or memory layout to show (the kernel test uses random "
               "inputs)")
# the recheck words of a captured GEMM alarm (ops.gemm.recheck_capture) and what each means here
RECHECK = {"output_wrong": "fault", "both_wrong": "fault", "weights_changed": "weights",
           "expected_wrong": "cleared", "not_reproduced": "cleared"}
STACK_KEYS = ("model", "precision", "checked", "torch", "cuda", "weights_digest", "version", "gpu")


def policy_with_defaults(p: Optional[dict]) -> dict:
    out = copy.deepcopy(DEFAULT_POLICY)
    for sec, vals in (p or {}).items():
        if sec not in out or not isinstance(vals, dict):
            raise ValueError(f"policy: unknown section {sec!r} (known: {', '.join(out)})")
        for k, v in vals.items():
            if k not in out[sec]:
                raise ValueError(f"policy: unknown key {sec}.{k}")
            out[sec][k] = v
    return out


@dataclass
class Section:
    name: str
    verdict: str
    effect: str                      # reject | missing | ok | info
    why: list = field(default_factory=list)
    detail: dict = field(default_factory=dict)

    def as_dict(self) -> dict:
        return {"verdict": self.verdict, "effect": self.effect, "why": self.why, **self.detail}


# ------------------------------------------------------------------------------------------ evidence readers
def _num(v) -> Optional[float]:
    return float(v) if isinstance(v, (int, float)) and v == v and abs(v) != float("inf") else None


def worker_coverage(metrics_texts: list) -> dict:
    """Per worker, what its /metrics say it checked (this package's server metrics)."""
    workers = []
    for text in metrics_texts:
        m = _client.parse_metrics(text)
        info = (m.get("sdcguard_protection_info{}") or [({}, 0)])[0][0]
        stack = (m.get("sdcguard_stack_info{}") or [({}, 0)])[0][0]
        wk = (m.get("sdcguard_worker_info{}") or [({}, 0)])[0][0]
        w = {k: _num(m.get(f"sdcguard_{k}")) for k in (
            "layers_checked", "layers_unchecked", "weights_checked_ratio", "checks_total", "polls_total",
            "alarms_total", "alerts_total", "confirmed_alerts_total", "fp8_layers_checked", "fp8_calls_judged_total",
            "fp8_findings_total", "weight_scan_entries", "weight_scan_passes_total", "weight_scan_never_compared",
            "weight_scan_changed", "weight_repairs_total", "weight_scan_left_out", "weight_scan_oldest_age_seconds",
            "protected")}
        w.update({"settings": info, "stack": stack, "gpu_uuid": wk.get("uuid")})
        workers.append(w)
    checked = bool(workers) and all((w["layers_checked"] or 0) > 0 and (w["checks_total"] or 0) > 0
                                    and (w["polls_total"] or 0) > 0 for w in workers)
    ratios = [w["weights_checked_ratio"] for w in workers]
    counted = [w["alerts_total"] for w in workers]
    return {"workers": workers, "checked": checked,
            "min_weights_checked": min(ratios) if ratios and None not in ratios else None,
            "alerts_counted": sum(counted) if counted and None not in counted else None,
            "checks": sum(w["checks_total"] or 0 for w in workers)}


def read_alerts(path: str) -> list:
    """The records of an alert log (JSONL); a line that is not a JSON object becomes {"unreadable": line number},
    so a cut or corrupted log shows instead of reading as fewer alerts."""
    out = []
    with open(path) as f:
        for k, line in enumerate(f, 1):
            if not line.strip():
                continue
            try:
                rec = json.loads(line)
            except ValueError:
                rec = None
            out.append(rec if isinstance(rec, dict) else {"unreadable": k})
    return out


@dataclass
class Witness:
    """What one arithmetic source showed: how much it tested, faults, open questions, notes."""
    name: str
    tested: int = 0
    faults: list = field(default_factory=list)
    unresolved: list = field(default_factory=list)
    notes: list = field(default_factory=list)
    summary: dict = field(default_factory=dict)
    not_a_source: Optional[str] = None          # why it cannot stand for "no fault", when it cannot


def _where(ev: dict) -> str:
    d = ev.get("detail") or {}
    return str(d.get("layer") or d.get("weight") or d.get("where") or "?")


def serving_witness(alerts: list, cov: Optional[dict], min_weights: Optional[float]) -> tuple:
    """The candidate server's alerts, judged by their own evidence, and its coverage. Returns (witness, weight
    findings, quantization findings)."""
    w = Witness("server_alerts")
    weights, quant = [], []
    counts = {"records": 0, "unreadable": 0, "confirmed_wrong": 0, "cleared": 0, "unconfirmed": 0}
    for ev in alerts:
        if "unreadable" in ev:
            counts["unreadable"] += 1
            continue
        counts["records"] += 1
        det, d = ev.get("detector"), ev.get("detail") or {}
        at = f" at step {ev['step']}" if ev.get("step") is not None else ""
        if det == "weights":
            weights.append({"where": _where(ev), "step": ev.get("step"), "repaired": d.get("repaired")})
            continue
        if det == "quantization":
            quant.append({"where": _where(ev), "step": ev.get("step")})
            continue
        if det in ("replay", "spot", "collective", "kv_transfer", "alltoall"):
            counts["confirmed_wrong"] += 1
            w.faults.append(f"{det} check on {_where(ev)}{at}: the recomputed result differs")
            continue
        if det == "runtime":
            counts["unconfirmed"] += 1
            w.unresolved.append(f"a kernel's bounded wait ran out{at} ({d.get('what')}): its checks were not judged")
            continue
        rv = (d.get("recheck") or {}).get("verdict")
        kind = RECHECK.get(rv)
        if kind == "fault":
            counts["confirmed_wrong"] += 1
            w.faults.append(f"alarm on {_where(ev)}{at}: its float64 recheck says {rv}")
        elif kind == "weights":
            weights.append({"where": _where(ev), "step": ev.get("step"), "repaired": None})
        elif kind == "cleared":
            counts["cleared"] += 1
            w.notes.append(f"alarm on {_where(ev)}{at}: the recheck cleared the output ({rv})")
        else:
            counts["unconfirmed"] += 1
            w.unresolved.append(f"alarm on {_where(ev)}{at}: recheck {rv or 'missing (no row captured)'}")
    w.summary = {**counts, "coverage": cov}
    gaps = []
    if counts["unreadable"]:
        gaps.append(f"{counts['unreadable']} lines of the alert log are not records")
    if cov is None:
        gaps.append("no worker metrics were given (--plugin-metrics)")
    else:
        if not cov["checked"]:
            gaps.append("a worker's metrics show no checked layer, no check run, or no result read back")
        if min_weights is not None and not ((cov["min_weights_checked"] or 0.0) >= min_weights):
            gaps.append(f"a worker checks {cov['min_weights_checked'] or 0:.0%} of the linear-layer weights, under "
                        f"the policy's {min_weights:.0%}")
        counted = cov["alerts_counted"]
        if counted is None:
            gaps.append("a worker's metrics do not say how many alerts it counted")
        elif counted > counts["records"]:
            gaps.append(f"the workers counted {counted:g} alerts but the log holds {counts['records']} (cut short or "
                        "lost)")
        elif counted < counts["records"]:
            w.notes.append(f"{counts['records']} alert records for {counted:g} counted in the metrics (alerts after "
                           "the metrics were read, or another run's records)")
        w.tested = int(cov["checks"]) if not gaps else 0
    if gaps:
        w.not_a_source = "; ".join(gaps)
    return w, weights, quant


GATE_JUDGED = ("PASSED", "FIXED", "REGRESSED", "UNCHANGED")


def gate_witness(gate: dict) -> Witness:
    """`gate compare` output ({"cases": {id: verdict record}} or a plain id -> record map)."""
    w = Witness("gate_cases")
    cases = gate.get("cases", gate) if isinstance(gate, dict) else {}
    seen: dict = {}
    for cid, v in cases.items():
        v = v if isinstance(v, dict) else {}
        word, why = v.get("verdict"), str(v.get("why", ""))[:160]
        seen[str(word)] = seen.get(str(word), 0) + 1
        if word in GATE_JUDGED:
            w.tested += 1
        if word == "REGRESSED" or (word == "UNCHANGED" and "avoided" not in why):
            w.faults.append(f"kept case {cid}: {word} ({why})")
        elif word == "UNCHANGED":
            w.notes.append(f"kept case {cid}: right on the candidate only because another kernel ran (avoided, not "
                           "fixed)")
        elif word not in ("PASSED", "FIXED"):
            w.unresolved.append(f"kept case {cid}: {word} ({why})")
    w.summary = {"cases": len(cases), "verdicts": seen, "judged": w.tested}
    if not w.tested:
        w.not_a_source = "the gate report judged no case on both stacks"
    return w


KERNEL_WORDS = ("PASSED", "WRONG", "OTHER KERNEL", "NOT RUN")


def kernel_test_witness(kt: dict) -> Witness:
    """`sdcguard kernels test` output: per call a verdict with its runs."""
    w = Witness("kernel_test")
    seen = dict.fromkeys(KERNEL_WORDS, 0)
    for row in kt.get("calls") or []:
        if not isinstance(row, dict):
            continue
        word, runs = row.get("verdict"), row.get("runs")
        if word not in seen:
            w.unresolved.append(f"kernel test: unknown verdict {word!r} for {row.get('call')}")
            continue
        seen[word] += 1
        ran = isinstance(runs, int) and runs > 0
        if word == "WRONG":
            w.faults.append(f"kernel test: {row.get('runs_wrong')} of {runs} runs wrong for {row.get('call')}")
        if word in ("PASSED", "WRONG") and not ran:
            w.unresolved.append(f"kernel test: {row.get('call')} is {word} with no run recorded")
        elif word == "PASSED" and row.get("runs_wrong"):
            w.unresolved.append(f"kernel test: {row.get('call')} PASSED with wrong runs")
        elif word in ("PASSED", "WRONG"):
            w.tested += 1
    stated = kt.get("counts") or {}
    want = dict(seen, **{"NOT RUN": seen["NOT RUN"] + len(kt.get("not_run") or [])})
    off = [k for k in set(stated) | set(want) if stated.get(k, 0) != want.get(k, 0)]
    if stated and off:
        w.unresolved.append("kernel test: its counts disagree with its rows (" + ", ".join(sorted(off)) + ")")
    if seen["OTHER KERNEL"]:
        w.notes.append(f"kernel test: {seen['OTHER KERNEL']} calls ran on another kernel here than in the workload")
    w.summary = {"counts": want, "judged": w.tested, "gpu": kt.get("gpu")}
    if not w.tested:
        w.not_a_source = "the kernel test judged no call on the workload's kernel"
    return w


# ------------------------------------------------------------------------------------------ sections
def arithmetic(witnesses: list) -> Section:
    faults = [f for w in witnesses for f in w.faults]
    unresolved = [u for w in witnesses for u in w.unresolved]
    notes = [n for w in witnesses for n in w.notes]
    counting = [w.name for w in witnesses if w.tested > 0 and w.not_a_source is None]
    empty = [f"{w.name}: {w.not_a_source}" for w in witnesses if w.not_a_source]
    detail = {"faults": faults, "unresolved": unresolved, "notes": notes, "sources_counting": counting,
              "sources": {w.name: {"tested": w.tested, "not_a_source": w.not_a_source, **w.summary}
                          for w in witnesses}}
    if faults:
        return Section("arithmetic", "FAULT", "reject", faults[:1] + ([f"and {len(faults) - 1} more"]
                                                                    if len(faults) > 1 else []), detail)
    if not witnesses:
        return Section("arithmetic", "INCONCLUSIVE", "missing", ["no arithmetic source was given"], detail)
    if not counting:
        return Section("arithmetic", "INCONCLUSIVE", "missing", (empty + unresolved)[:3], detail)
    if unresolved:
        return Section("arithmetic", "INCONCLUSIVE", "missing", unresolved[:3], detail)
    return Section("arithmetic", "NO FAULT OBSERVED", "ok", [f"tested by {', '.join(counting)}"] + empty, detail)


def weights(findings: list, cov: Optional[dict], alerts_given: bool) -> Section:
    if findings:
        names = sorted({f["where"] for f in findings})
        steps = [f["step"] for f in findings if f.get("step") is not None]
        repaired = sum(1 for f in findings if f.get("repaired"))
        why = (f"the weights of {', '.join(names[:3])}" + (f" and {len(names) - 3} more" if len(names) > 3 else "")
               + " changed since load" + (f" (first at step {min(steps)})" if steps else "")
               + (f"; {repaired} written back from the host copy, after requests may have used them" if repaired
                  else "") + ": a corrupted or overwritten weight, whatever the arithmetic did with it")
        return Section("weights", "CHANGED", "reject", [why], {"layers": names, "findings": len(findings)})
    workers = (cov or {}).get("workers") or []
    changed = sum(w.get("weight_scan_changed") or 0 for w in workers)
    repairs = sum(w.get("weight_repairs_total") or 0 for w in workers)
    if changed or repairs:
        return Section("weights", "CHANGED", "reject",
                       [f"the weight scan counts {changed:g} changed entries and {repairs:g} repairs (their alert "
                        "records are not in the log given)"])
    if cov is None or not alerts_given:
        return Section("weights", "UNMEASURED", "info",
                       ["no worker metrics given" if cov is None else "no alert log given"])
    scanned = [w for w in workers if (w.get("weight_scan_entries") or 0) > 0]
    if workers and len(scanned) == len(workers) and all(
            w.get("weight_scan_never_compared") == 0 and w.get("weight_scan_oldest_age_seconds") is not None
            for w in workers):
        age = max(w["weight_scan_oldest_age_seconds"] for w in workers)
        entries = sum(w["weight_scan_entries"] for w in workers)
        left = sum(w.get("weight_scan_left_out") or 0 for w in workers)
        return Section("weights", "VERIFIED", "info",
                       [f"the weight scan compared all {entries:g} entries on every worker with their fingerprints "
                        f"at load and found no change; the least recently verified was clean {age:.0f} s before the "
                        f"metrics were read; {left:g} tensors left out"],
                       {"entries": entries, "oldest_verification_age_seconds": age, "left_out": left})
    why = ("no weight scan ran (--weight-scan-mb)" if not scanned else
           "the weight scan has not compared every entry on every worker yet")
    if cov.get("checked"):
        return Section("weights", "NO CHANGE SEEN", "info",
                       [f"no alert showed a changed weight, but {why}; the ABFT checksums see a changed weight only "
                        "once it moves an output past their line"])
    return Section("weights", "UNMEASURED", "info", [why + ", and the metrics show no checks that ran"])


def quantization(findings: list, cov: Optional[dict]) -> Section:
    if findings:
        names = sorted({f["where"] for f in findings})
        return Section("quantization", "WRONG", "reject",
                       [f"fp8 activation quantization differed from its replay on {', '.join(names[:3])}"
                        + (f" and {len(names) - 3} more" if len(names) > 3 else "")], {"layers": names})
    workers = (cov or {}).get("workers") or []
    if any((w.get("fp8_findings_total") or 0) > 0 for w in workers):
        return Section("quantization", "WRONG", "reject",
                       ["the workers' metrics count fp8 quantization findings not in the alert log"])
    judged = [w.get("fp8_calls_judged_total") or 0 for w in workers]
    if workers and all(j > 0 for j in judged):
        return Section("quantization", "RIGHT", "info",
                       [f"the fp8 quantization replays judged {sum(judged):g} calls and found nothing"],
                       {"calls_judged": sum(judged)})
    return Section("quantization", "UNMEASURED", "info",
                   ["no fp8 layers, or no worker metrics given" if workers or cov is None else "no workers"])


def approximation(quality: Optional[dict], pol: dict) -> Section:
    if quality is None:
        return Section("approximation", "UNMEASURED", "missing", ["no model-check was given"])
    v = quality.get("verdict")
    if isinstance(v, dict):                    # a nested verdict record
        v = v.get("verdict")
    q = pol["quality"]
    s = {k: quality.get(k) for k in ("mean_kl", "top1_agreement", "worst_prompt_kl", "positions")}
    if v not in ("PASS", "WARN", "FAIL"):
        return Section("approximation", "UNMEASURED", "missing", [f"the model-check was {v or 'unreadable'}"], s)
    extra = []
    if q["max_mean_kl"] is not None and not ((s["mean_kl"] if s["mean_kl"] is not None else float("inf"))
                                             <= q["max_mean_kl"]):
        extra.append(f"mean KL {s['mean_kl']} above the policy's {q['max_mean_kl']}")
    if q["min_top1"] is not None and not ((s["top1_agreement"] if s["top1_agreement"] is not None else -1.0)
                                          >= q["min_top1"]):
        extra.append(f"top-1 agreement {s['top1_agreement']} below the policy's {q['min_top1']}")
    if quality.get("alarms"):
        extra.append(f"the model-check's own run raised {quality['alarms']} alarms")
    if v == "FAIL" or extra or (v == "WARN" and not q["accept_warn"]):
        why = extra or ([f"model-check {v}"] if v == "FAIL" else ["model-check WARN, and the policy does not accept "
                                                                  "WARN"])
        return Section("approximation", "OUTSIDE", "reject", why, dict(s, check=v))
    return Section("approximation", "WITHIN", "ok", [f"model-check {v}: mean KL {s['mean_kl']}, top-1 "
                                                     f"{s['top1_agreement']}"], dict(s, check=v))


def performance(before: Optional[dict], after: Optional[dict], pol: dict) -> Section:
    p = pol["performance"]
    req = bool(p["required"])
    miss_effect, gap_effect = ("reject", "missing") if req else ("info", "info")
    if before is None or after is None:
        return Section("performance", "UNMEASURED", gap_effect, ["no pair of perf runs was given"], {"required": req})
    from .perf import compare
    c = compare(before, after)
    if not c["comparable"]:
        return Section("performance", "UNMEASURED", gap_effect, c["why"], {"required": req})
    m = c["metrics"]
    tp = m.get("output_tokens_per_s")
    if tp is None:
        return Section("performance", "UNMEASURED", gap_effect, ["no throughput in one of the runs"],
                       {"required": req})
    misses, unread = [], []
    g = p["min_throughput_gain"]
    if g is not None:
        if g > 0 and tp["change"] >= g and tp["noise"]:
            misses.append(f"throughput {tp['change']:+.1%} is within the noise ({tp['noise_band']:.1%}): the gain "
                          "is not shown")
        elif tp["change"] < g and not (g <= 0 and tp["noise"]):
            misses.append(f"throughput {tp['change']:+.1%}, the policy asks for at least {g:+.1%}")
    for key, metric in (("max_ttft_p99_increase", "ttft_p99_ms"), ("max_itl_p99_increase", "itl_p99_ms")):
        lim = p[key]
        if lim is None:
            continue
        x = m.get(metric)
        if x is None:
            unread.append(f"{metric} is limited by the policy and missing from a run")
        elif x["change"] > lim and not x["noise"]:
            misses.append(f"{metric} rose {x['change']:+.1%}, past the policy's {lim:+.1%}")
    detail = {"required": req, "metrics": m}
    if misses:
        return Section("performance", "MISSES", miss_effect, misses, detail)
    if unread:
        return Section("performance", "UNMEASURED", gap_effect, unread, detail)
    return Section("performance", "MEETS", "ok", [f"throughput {tp['change']:+.1%}"
                                                  + (" (within noise)" if tp["noise"] else "")], detail)


def isolation(iso: Optional[dict], pol: dict) -> Section:
    req = bool(pol["isolation"]["required"])
    if iso is None or iso.get("verdict") not in ("LEAK", "NO LEAK SEEN"):
        why = "no isolation check was given" if iso is None else f"the isolation check was {iso.get('verdict')}"
        return Section("isolation", "UNMEASURED", "missing" if req else "info",
                       [why] + list((iso or {}).get("why") or [])[:2], {"required": req})
    v = iso["verdict"]
    return Section("isolation", v, "reject" if v == "LEAK" else "ok",
                   list(iso.get("why") or []) or ["no probe's answer depended on another request"],
                   {"required": req, "primer": iso.get("primer")})


def consistency(cons: Optional[dict], base: Optional[dict], pol: dict) -> Section:
    req = bool(pol["consistency"]["required"])
    if cons is None:
        return Section("consistency", "UNMEASURED", "missing" if req else "info",
                       ["no consistency check was given"], {"required": req})
    from .consistency import judge_against
    j = judge_against(cons, base)
    detail = {"required": req, "largest_gap": cons.get("largest_gap"),
              "baseline_largest_gap": (base or {}).get("largest_gap")}
    if j["verdict"] not in ("CONSISTENT", "INCONSISTENT"):
        return Section("consistency", "UNMEASURED", "missing" if req else "info", j["why"], detail)
    return Section("consistency", j["verdict"], "reject" if j["verdict"] == "INCONSISTENT" else "ok", j["why"],
                   detail)


def fingerprint(stack: Optional[dict]) -> str:
    """The parts of a stack a decision depends on, hashed: another value of any of them and the decision no longer
    applies as made."""
    blob = json.dumps({k: (stack or {}).get(k) for k in STACK_KEYS}, sort_keys=True, default=str)
    return hashlib.sha256(blob.encode()).hexdigest()[:16]


def scope(stacks: dict, kernels_before: Optional[dict], kernels_after: Optional[dict],
          kernel_test: Optional[dict], settings: Optional[dict]) -> dict:
    out: dict = {"stacks": stacks, "settings": settings, "not_checked": list(NOT_CHECKED),
                 "fingerprint": fingerprint(stacks.get("candidate")), "kernels": None}
    if kernels_before is not None and kernels_after is not None:
        from .kernels import diff
        d = diff(kernels_before, kernels_after)
        after = kernels_after.get("kernels") or {}
        out["kernels"] = {"added": d["only_after"], "dropped": d["only_before"], "kept": d["both"],
                          "work_share_on_added": d["work_moved"]}
        out["added_kernels_with_known_issues"] = [{"kernel": k, "issues": after[k].get("flags")}
                                                  for k in d["only_after"] if after.get(k, {}).get("flags")]
        tested = {str(r.get("kernel") or r.get("call", "")).split(" | ")[0]
                  for r in (kernel_test or {}).get("calls") or [] if isinstance(r, dict) and r.get("runs")}
        out["added_kernels_not_tested"] = [k for k in d["only_after"] if k not in tested]
    return out


# ------------------------------------------------------------------------------------------ the decision
def decide(pol: Optional[dict] = None, quality: Optional[dict] = None, gate: Optional[dict] = None,
           kernels_before: Optional[dict] = None, kernels_after: Optional[dict] = None,
           kernel_test: Optional[dict] = None, alerts: Optional[list] = None, perf_before: Optional[dict] = None,
           perf_after: Optional[dict] = None, metrics: Optional[list] = None, isolation_run: Optional[dict] = None,
           consistency_run: Optional[dict] = None, consistency_baseline: Optional[dict] = None,
           baseline_stack: Optional[dict] = None) -> dict:
    pol = policy_with_defaults(pol)
    cov = worker_coverage(metrics) if metrics is not None else None
    witnesses, wfind, qfind = [], [], []
    if alerts is not None or cov is not None:
        w, wfind, qfind = serving_witness(alerts or [], cov, pol["arithmetic"]["min_weights_checked"])
        if alerts is None:
            w.not_a_source = "no alert log was given" + (f"; {w.not_a_source}" if w.not_a_source else "")
            w.tested = 0
        witnesses.append(w)
    if gate is not None:
        witnesses.append(gate_witness(gate))
    if kernel_test is not None:
        witnesses.append(kernel_test_witness(kernel_test))
    secs = [arithmetic(witnesses), weights(wfind, cov, alerts is not None), quantization(qfind, cov),
            approximation(quality, pol), performance(perf_before, perf_after, pol), isolation(isolation_run, pol),
            consistency(consistency_run, consistency_baseline, pol)]
    reject = [f"{s.name}: {s.why[0] if s.why else s.verdict}" for s in secs if s.effect == "reject"]
    missing = [f"{s.name}: {'; '.join(s.why[:2]) or s.verdict}" for s in secs if s.effect == "missing"]
    if reject:
        d, why = "REJECT", reject
    elif missing:
        d, why = "NOT DECIDED", missing
    else:
        d, why = "ACCEPT", ["no reason to reject was found within the scope listed"]
    cand_stack = None
    if cov and cov["workers"]:
        cand_stack = dict(cov["workers"][0]["stack"] or {})
        cand_stack.setdefault("gpu", cov["workers"][0].get("gpu_uuid"))
    settings = [w["settings"] for w in cov["workers"]] if cov else None
    out = {"schema": SCHEMA, "decision": d, "why": why, **{s.name: s.as_dict() for s in secs},
           "scope": scope({"baseline": baseline_stack, "candidate": cand_stack}, kernels_before, kernels_after,
                          kernel_test, settings[0] if settings else None),
           "policy": pol, "created": time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime()), "created_unix": time.time()}
    return out


def still_applies(decision: dict, stack_now: Optional[dict]) -> dict:
    """Is stack_now (a server's stack record) the stack the decision was made on?"""
    was = ((decision.get("scope") or {}).get("stacks") or {}).get("candidate")
    if not was:
        return {"applies": None, "differences": [], "why": "the decision does not record the stack it was made on"}
    if not stack_now:
        return {"applies": None, "differences": [], "why": "the server publishes no stack record"}
    diffs = [f"{k}: {was.get(k)!r} then, {stack_now.get(k)!r} now" for k in STACK_KEYS
             if k in was and was.get(k) != stack_now.get(k)]
    return {"applies": not diffs, "differences": diffs,
            "why": "the stack is the one the decision was made on" if not diffs else
                   "the stack changed since the decision: " + "; ".join(diffs)}


def render(r: dict) -> str:
    """The decision as text a person reads first."""
    lines = [f"DECISION: {r['decision']}"] + [f"  {w}" for w in r["why"]] + [""]
    titles = [("arithmetic", "1. Arithmetic (against recomputation)"), ("weights", "1a. Weight integrity"),
              ("quantization", "1b. FP8 quantization"), ("approximation", "2. Approximation (model outputs)"),
              ("performance", "3. Performance"), ("isolation", "4. Isolation"),
              ("consistency", "4b. Consistency (decode vs prefill)")]
    for key, title in titles:
        s = r[key]
        req = s.get("required")
        lines.append(f"{title}: {s['verdict']}" + ("" if req is None else " (required)" if req else
                                                   " (not required)"))
        lines += [f"   {w}" for w in s.get("why") or []][:4]
        if key == "arithmetic":
            lines += [f"   unresolved: {u}" for u in s.get("unresolved", [])[:3]]
            lines += [f"   note: {n}" for n in s.get("notes", [])[:3]]
        if key == "performance":
            for m, x in (s.get("metrics") or {}).items():
                if x:
                    lines.append(f"   {m}: {x['baseline']} -> {x['candidate']} ({x['change']:+.1%}, "
                                 f"{x['direction']}" + (", within noise" if x["noise"] else "") + ")")
    sc = r["scope"]
    lines.append(f"5. Scope (candidate stack fingerprint {sc['fingerprint']})")
    for side in ("baseline", "candidate"):
        st = (sc.get("stacks") or {}).get(side)
        if st:
            lines.append(f"   {side}: " + ", ".join(f"{k} {st[k]}" for k in STACK_KEYS if st.get(k)))
    if sc.get("kernels"):
        k = sc["kernels"]
        lines.append(f"   kernels added {len(k['added'])}, dropped {len(k['dropped'])}, kept {k['kept']}")
        for x in sc.get("added_kernels_with_known_issues") or []:
            lines.append(f"   added, matches a known issue ({', '.join(x['issues'])}): {x['kernel']}")
        if sc.get("added_kernels_not_tested"):
            lines.append(f"   added kernels no test ran: {len(sc['added_kernels_not_tested'])}")
    lines += [f"   not checked: {n}" for n in sc["not_checked"]]
    return "\n".join(lines)


def applies(decision: dict, url: str) -> dict:
    m = _client.scrape(url)
    if m is None:
        return {"applies": None, "differences": [], "why": f"no metrics at {url}"}
    rows = m.get("sdcguard_stack_info{}") or []
    stack = dict(rows[0][0]) if rows else None
    wk = (m.get("sdcguard_worker_info{}") or [({}, 0)])[0][0]
    if stack is not None:
        stack.setdefault("gpu", wk.get("uuid"))
    return still_applies(decision, stack)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="sdcguard decide", description=__doc__.split("\n\n")[0])
    ap.add_argument("--policy")
    ap.add_argument("--quality")
    ap.add_argument("--gate")
    ap.add_argument("--kernels", nargs=2, metavar=("BEFORE", "AFTER"))
    ap.add_argument("--kernel-test")
    ap.add_argument("--alerts")
    ap.add_argument("--plugin-metrics", nargs="+", metavar="METRICS")
    ap.add_argument("--perf", nargs=2, metavar=("BEFORE", "AFTER"))
    ap.add_argument("--isolation")
    ap.add_argument("--consistency", nargs="+", metavar="RUN")
    ap.add_argument("--out")
    ap.add_argument("--json", action="store_true")
    ap.add_argument("--applies", metavar="DECISION")
    ap.add_argument("--url", default="http://127.0.0.1:8000")
    a = ap.parse_args(argv)

    def ld(p):
        if not p:
            return None
        with open(p) as f:
            return json.load(f)

    if a.applies:
        r = applies(ld(a.applies), a.url)
        print(r["why"])
        return {True: 0, False: 1}.get(r["applies"], 2)
    metrics = None
    if a.plugin_metrics:
        metrics = []
        for p in a.plugin_metrics:
            with open(p) as f:
                metrics.append(f.read())
    kb, ka = (ld(a.kernels[0]), ld(a.kernels[1])) if a.kernels else (None, None)
    pb, pa = (ld(a.perf[0]), ld(a.perf[1])) if a.perf else (None, None)
    r = decide(ld(a.policy), ld(a.quality), ld(a.gate), kb, ka, ld(a.kernel_test),
               read_alerts(a.alerts) if a.alerts else None, pb, pa, metrics, ld(a.isolation),
               ld(a.consistency[0]) if a.consistency else None,
               ld(a.consistency[1]) if a.consistency and len(a.consistency) > 1 else None)
    if a.out:
        with open(a.out, "w") as f:
            json.dump(r, f, indent=1, default=str)
        with open(os.path.splitext(a.out)[0] + ".txt", "w") as f:
            f.write(render(r) + "\n")
    print(json.dumps(r, indent=1, default=str) if a.json else render(r))
    return {"ACCEPT": 0, "REJECT": 1}.get(r["decision"], 2)


if __name__ == "__main__":
    raise SystemExit(main())
