"""Coverage gate for recordings of this package's own prefill/decode engine (`sdcguard_b200.serve.pd`).

The per-request semantics are those of the recorded-vLLM gate, applied to the same record schema: each request
needs exactly one `recv_plan` and one `verification` record; the verification's chunk scope is re-derived from its
primitive observations (`observer.classify_verification`), never read from stored verdict fields, and stored
derived fields that disagree hold the request. A request passes only if every chunk of its prompt was compared
and matched. Chunks served from the consumer's prefix cache count as compared only when a
`cached_prefix_verification` record shows them re-hashed against this request's producer checksums; otherwise
the request holds with the reference's reason, "cached prefix not covered by checksum".

Output keeps the full-prompt gate's text layout (`gate.render`) and exit codes (0 PASS, 2 HOLD).
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

from . import evidence as ev
from . import gate
from . import observer as obs

PLAN_SCHEMA = "sdcguard_b200.pd-request-plan.v1"


def _files(path: Path) -> dict:
    names = ("RESULT.json", "REQUEST_PLAN.json", "OBSERVER.json", "CACHE.json", "CACHED_PREFIX_VERIFICATION.json")
    return {n: ev.read_file(path, n) for n in names}


def evaluate(files: dict) -> dict:
    result = ev.parse_json(files["RESULT.json"])
    issues = []
    for name, raw in files.items():
        if name != "RESULT.json" and result.get("files_sha256", {}).get(name) != ev.digest(raw):
            issues.append("recording_file_digest_disagrees:" + name)
    plan = ev.parse_json(files["REQUEST_PLAN.json"])
    snap = ev.parse_json(files["OBSERVER.json"])
    cache = ev.parse_json(files["CACHE.json"])
    pver = ev.parse_json(files["CACHED_PREFIX_VERIFICATION.json"])
    if plan.get("schema") != PLAN_SCHEMA or snap.get("schema") != obs.SCHEMA or cache.get("schema") != obs.CACHE_SCHEMA:
        raise ev.EvidenceError("unsupported recording schema")
    if snap.get("closed") is not True or snap.get("health", {}).get("complete") is not True:
        issues.append("observer_not_closed_or_incomplete")
    recs = snap.get("records", [])
    by_req: dict = {}
    for r in recs:
        if type(r) is dict and type(r.get("request_id")) is str:
            by_req.setdefault(r["request_id"], []).append(r)
    seqs = [r.get("sequence") for r in recs if type(r) is dict]
    if seqs != sorted(seqs) or len(set(seqs)) != len(seqs):
        issues.append("record_order_unverified")
    decode_cache = {r["request_id"]: r for r in cache.get("records", []) if r.get("role") == "decode"}
    prefill_cache = {r["request_id"]: r for r in cache.get("records", []) if r.get("role") == "prefill"}
    reverified = {r["request_id"]: r for r in pver.get("records", [])}
    rows = []
    planned = {q["request_id"] for q in plan.get("requests", [])}
    for rid in by_req:
        if rid not in planned:
            issues.append("unplanned_native_transfer_record")
    for q in plan.get("requests", []):
        rid, n = q["request_id"], q["prompt_tokens"]
        reasons: list[str] = []
        rr = by_req.get(rid, [])
        plans = [r for r in rr if r.get("kind") == "recv_plan"]
        vers = [r for r in rr if r.get("kind") == "verification"]
        tc = {"prompt_tokens": n, "transferred_tokens_checked": None, "decode_cached_tokens_unchecked": None,
              "prefill_cached_tokens": None}
        check = {"native_result": "unverified", "expected_units": None, "compared_units": None, "completed": False,
                 "evidence_complete": False, "applicable": True, "reason": None}
        if len(plans) != 1 or len(vers) != 1:
            reasons.append("unambiguous_native_checksum_call_missing")
        else:
            v = vers[0]
            d = obs.classify_verification(v)
            for k, want in d.items():
                if k in v and not ev.same(v[k], want):
                    reasons.append("derived_observation_disagrees:" + k)
            if not obs.plan_matches_proof(plans[0], v.get("proof", {})):
                reasons.append("planned_chunk_scope_disagrees_with_verification")
            proof = v.get("proof", {})
            if proof.get("num_tokens") != n:
                reasons.append("client_prompt_to_checksum_span_unverified")
            compared = list(d["compared_units"] or [])
            other = [x for x in d["reasons"] if x != obs.CACHED_PREFIX_REASON]
            reasons.extend(other)
            local = proof.get("num_local_computed_tokens")
            if d["native_result"] == "mismatch":
                reasons.append("native_checksum_mismatch")
            if type(local) is int and local > 0 and not other:
                pv = reverified.get(rid)
                want = [f"group:0:chunk:{c}" for c in range(local // 16)]
                if pv is not None and pv.get("compared_units") == want and pv.get("mismatched_units") == []:
                    compared = want + compared
                elif pv is not None and pv.get("mismatched_units"):
                    reasons.append("cached_prefix_checksum_mismatch")
                else:
                    reasons.append(obs.CACHED_PREFIX_REASON)
            dc = decode_cache.get(rid, {}).get("stats") or {}
            if type(local) is int:
                checked_cached = local if not any(r == obs.CACHED_PREFIX_REASON for r in reasons) else 0
                tc.update(transferred_tokens_checked=(n - local) if not other else None,
                          decode_cached_tokens_unchecked=local - checked_cached)
            if dc and dc.get("num_local_cached_tokens") != local:
                reasons.append("native_cache_to_checksum_span_unverified")
            pc = prefill_cache.get(rid, {}).get("stats") or {}
            tc["prefill_cached_tokens"] = pc.get("num_local_cached_tokens")
            ok = not reasons and d["expected_units"] is not None and compared == d["expected_units"]
            check.update(native_result=d["native_result"], expected_units=d["expected_units"],
                         compared_units=compared if compared else None, completed=ok, evidence_complete=ok,
                         reason=reasons[0] if reasons else "complete_recorded_comparison")
        rows.append(dict(client_request_id=rid, arm_id="pd", slot=len(rows), checks={"checksum": check},
                         token_coverage=tc, reasons=list(dict.fromkeys(reasons))))
    ans = gate.decide(rows, ["checksum"], issues, total=len(rows),
                      engine={"name": "sdcguard_b200", "version": plan.get("engine_version", "unknown"),
                              "source_profile": plan.get("source_profile")})
    if any(r["decision"] == "HOLD" for r in ans["requests"]):
        ans["decision"] = "HOLD"
        ans["hold_reasons"].insert(0, gate.COVERAGE_HOLD)
    return ans


def inspect(path) -> dict:
    path = Path(path)
    files = _files(path)
    ans = evaluate(files)
    if _files(path) != files:
        raise ev.EvidenceError("recording changed during inspection")
    return ans


def is_own_recording(path) -> bool:
    p = Path(path)
    return (p / "REQUEST_PLAN.json").is_file() and (p / "OBSERVER.json").is_file()


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="sdcguard gate (sdcguard_b200 recording)")
    ap.add_argument("input")
    ap.add_argument("--json", action="store_true")
    a = ap.parse_args(argv)
    try:
        ans = inspect(a.input)
    except (ValueError, OSError, KeyError, TypeError, AttributeError) as e:
        ans = gate.decide([], ["checksum"], ["evidence_unverifiable:" + str(e)])
    sys.stdout.write(ev.json_bytes(ans).decode() if a.json else gate.render(ans))
    return 0 if ans["decision"] == "PASS" else 2
