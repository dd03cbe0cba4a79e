"""Offline interpretation of recorded KV-checksum observations.

A recording holds, per decode engine, a closed snapshot (`sdcguard.checksum-observer.v1`) of two record kinds:
`recv_plan` (what the consumer planned to receive and compare: token count, locally cached prefix, block groups,
the producer's checksum array shape and fingerprint) and `verification` (the native comparison call: its return,
per-group witnesses, and the proof of scope). From these the gate re-derives, never trusting a stored verdict:

    expected units   group:G:chunk:i  for every 16-token chunk of the prompt
    compared units   the chunks from the first transferred chunk on, when the comparison is established
    coverage         complete | partial (cached prefix not compared) | not_covered | unknown
    token coverage   prompt tokens, transferred tokens checked, decode-cache tokens reused unchecked

and the prefill-accounting snapshot (`sdcguard.native-prefill-accounting.v1`) gives per-request cache counts.

The decision table follows the record semantics of the reference recorder (src/sdcguard/kv_checksum_observer.py:
133-330 `classify_verification`, :84-130 engine-pass gap reasons; checksum_observer_report.py:70-246;
prefix_cache_observer.py:246-313), because the verdicts must agree for the same recordings; the implementation is
this package's own. This package's own P/D engine writes records of the same schema (sdcguard_b200.serve.pd).
"""
from __future__ import annotations

import json
from collections import Counter

from . import evidence as ev
from . import profiles

SCHEMA = "sdcguard.checksum-observer.v1"
CACHE_SCHEMA = "sdcguard.native-prefill-accounting.v1"
CACHED_PREFIX_REASON = "cached prefix not covered by checksum"
CALL_PATH = ["on_new_request", "add_recv", "update_from_output", "_verify", "_compare_group"]
MAX_GROUPS = 16
MAX_RECORDS = 4096
MAX_UNITS = 65536
FIXED_METADATA_BYTES = 16384
CACHE_MAX_RECORDS = 16384
CACHE_MAX_BYTES = 8 * 1024 * 1024
CACHE_FIXED_BYTES = 8192
MAX_PROMPT_TOKENS = 8192
CACHE_FIELDS = ("num_prompt_tokens", "num_computed_tokens", "num_cached_tokens", "num_local_cached_tokens",
                "num_external_cached_tokens")
CACHE_STATUSES = ("WAITING", "WAITING_FOR_STRUCTURED_OUTPUT_GRAMMAR", "WAITING_FOR_REMOTE_KVS",
                  "WAITING_FOR_STREAMING_REQ", "RUNNING", "PREEMPTED", "FINISHED_STOPPED", "FINISHED_LENGTH_CAPPED",
                  "FINISHED_ABORTED", "FINISHED_IGNORED", "FINISHED_ERROR", "FINISHED_REPETITION")
FINISHED_OK = ("FINISHED_STOPPED", "FINISHED_LENGTH_CAPPED")


def _int(v, lo=0, hi=2 ** 63 - 1) -> bool:
    return type(v) is int and lo <= v <= hi


def _u64(v) -> bool:
    return type(v) is int and 0 <= v < 2 ** 64


def _text(v, n=1024) -> bool:
    return type(v) is str and 0 < len(v) <= n and "\x00" not in v


def _shape(v, want) -> bool:
    return type(v) is list and len(v) == len(want) and all(type(x) is int and x == y for x, y in zip(v, want))


def _prim_same(a, b) -> bool:
    try:
        return json.dumps(a, sort_keys=True, allow_nan=False) == json.dumps(b, sort_keys=True, allow_nan=False)
    except (ValueError, TypeError):
        return False


def _gap_reasons(record: dict, proof: dict) -> list[str]:
    """Native passes that still leave chunks uncompared: empty replica inputs, or a compared span that does
    not line up with the producer's span."""
    if (record.get("native_return") is not True or proof.get("source_supported") is not True
            or proof.get("metadata_stable") is not True or record.get("engine_exception") is not None
            or record.get("unverified_reasons") != []):
        return []
    groups, wit = proof.get("groups"), record.get("groups")
    if (type(groups) is not list or len(groups) != 1 or type(groups[0]) is not dict
            or type(wit) is not list or len(wit) != 1 or type(wit[0]) is not dict):
        return []
    g, w = groups[0], wit[0]
    if (g.get("compare_called") is not True or g.get("native_group_result") != []
            or g.get("native_group_error") is not None or w.get("native_result") != "passed"
            or w.get("returned_positions") != [] or w.get("reason") is not None
            or not _int(g.get("group_id")) or type(w.get("group_id")) is not int or w["group_id"] != g["group_id"]):
        return []
    out = []
    count, reps = g.get("block_count"), g.get("consumer_reports")
    if _int(count, 1) and type(reps) is list and len(reps) == 1 and type(reps[0]) is dict:
        r = reps[0]
        if type(r.get("replica_keys")) is list and r.get("replica_keys") == [] and _shape(r.get("value_shape"),
                                                                                          [count, 0]):
            out.append("empty_replica_inputs")
    bs, sbs = g.get("block_size"), g.get("sent_block_size")
    start, sstart, scount = g.get("start"), g.get("sent_start"), g.get("sent_count")
    nt, et = proof.get("num_tokens"), proof.get("expected_num_tokens")
    if (g.get("spec_type") != "FullAttentionSpec" or g.get("spec_source_supported") is not True
            or not _int(bs, 1) or type(sbs) is not int or bs != sbs or not _int(start) or not _int(sstart)
            or not _int(count, 1) or not _int(scount, 1) or not _int(nt, 1) or not _int(et, 1)
            or count != (nt + bs - 1) // bs - start or scount != (et + bs - 1) // bs - sstart
            or not _shape(g.get("sent_shape"), [scount])):
        return out
    lo, hi = max(start, sstart), min(start + count, sstart + scount)
    if lo < hi:
        partial = lo > start or hi < start + count
        for pos in {(nt - 1) // bs, (et - 1) // bs}:      # only a last chunk can hold different token counts
            if lo <= pos < hi:
                partial = partial or min(bs, max(0, nt - pos * bs)) != min(bs, max(0, et - pos * bs))
        if partial:
            out.append("partial_checksum_span")
    return out


def classify_verification(record, *, max_units: int = MAX_UNITS) -> dict:
    """Re-derive the conditional chunk scope of one `verification` record from its primitive observations."""
    if not _int(max_units, 1) or max_units > 1048576:
        raise ValueError("max_units must be between 1 and 1048576")
    rec = record if type(record) is dict else {}
    native = rec.get("native_return") if type(rec.get("native_return")) is bool else None
    res = {"native_return": native, "native_result": "passed" if native is True else "unverified",
           "expected_units": None, "compared_units": None, "missing_units": None, "coverage": "unknown",
           "reason": "scope_metadata_unverified", "reasons": [],
           "token_coverage": {"prompt_tokens": None, "transferred_tokens_checked": None,
                              "decode_cached_tokens_unchecked": None}}
    R: list[str] = []
    proof = rec.get("proof") if type(rec.get("proof")) is dict else {}
    if proof.get("scope_budget_refused") is True:
        R.append("scope_budget_refused")
    groups = proof.get("groups") if type(proof.get("groups")) is list else []
    unv = rec.get("unverified_reasons", [])
    if type(unv) is not list or len(unv) > MAX_GROUPS or any(type(x) is not str or len(x) > 512 for x in unv):
        R.append("native_unverified_reason_shape_invalid")
    elif unv:
        R.append("native_comparison_unverified")
    if rec.get("engine_exception") is not None:
        R.append("native_engine_exception_present")
    path = proof.get("call_path")
    if path != CALL_PATH or not _int(rec.get("origin_update_sequence"), 1) or not _int(proof.get("plan_sequence"), 1):
        R.append("native_call_path_unverified")
    if proof.get("source_supported") is not True:
        R.append("source_profile_unverified")
    if proof.get("metadata_stable") is not True:
        R.append("scope_metadata_changed_or_unobserved")
    par = proof.get("parallel")
    if (type(par) is not dict or any(not _int(par.get(k), 1) or par[k] != 1 for k in ("tp", "pp", "dp", "dcp", "pcp"))
            or type(proof.get("num_workers")) is not int or proof.get("num_workers") != 1
            or type(proof.get("native_tp_size")) is not int or proof.get("native_tp_size") != 1):
        R.append("parallel_scope_unsupported")
    if proof.get("speculative_disabled") is not True:
        R.append("speculative_configuration_unknown_or_enabled")
    if proof.get("producer_payload_present") is not True:
        R.append("producer_checksum_payload_missing_or_unverified")
    local, nt, et = proof.get("num_local_computed_tokens"), proof.get("num_tokens"), proof.get("expected_num_tokens")
    if not _int(local) or not _int(nt, 1) or local >= nt:
        R.append("local_prefix_scope_unsupported")
    if not _int(nt, 1) or type(et) is not int or nt != et:
        R.append("producer_consumer_token_scope_differs")
    if (type(proof.get("expected_tp_size")) is not int or proof.get("expected_tp_size") != 1
            or type(proof.get("planned_group_count")) is not int or proof.get("planned_group_count") != 1
            or type(proof.get("configured_group_count")) is not int or proof.get("configured_group_count") != 1
            or len(groups) != 1):
        R.append("group_scope_unsupported")
    ranks = proof.get("worker_ranks")
    if not (type(ranks) is list and len(ranks) == 1 and _shape(ranks[0], [0, 0])
            and type(proof.get("worker_report_count")) is int and proof["worker_report_count"] == 1):
        R.append("worker_rank_scope_unverified")
    expected: list = []
    compared = None
    established = False
    if len(groups) == 1 and type(groups[0]) is dict:
        g = groups[0]
        gid, bs, count = g.get("group_id"), g.get("block_size"), g.get("block_count")
        if (proof.get("scope_budget_refused") is True or not _int(gid) or not _int(bs, 1) or not _int(count, 1)
                or count > max_units // 2):
            R.append("chunk_scope_budget_or_shape_invalid")
        else:
            full = (nt + bs - 1) // bs if _int(nt, 1) else None
            coord = (g.get("spec_type") == "FullAttentionSpec" and g.get("spec_source_supported") is True
                     and _int(local) and _int(nt, 1) and local < nt and local % bs == 0
                     and type(g.get("start")) is int and g["start"] == local // bs
                     and type(g.get("sent_block_size")) is int and g["sent_block_size"] == bs
                     and full <= max_units // 2)
            if coord:
                expected = [f"group:{gid}:chunk:{i}" for i in range(full)]
            else:
                R.append("local_prefix_coordinate_scope_unverified")
            if (g.get("spec_type") != "FullAttentionSpec" or g.get("spec_source_supported") is not True
                    or g.get("sliding_window") is not None or g.get("attention_chunk_size") is not None
                    or g.get("non_causal") is not False or g.get("spec_fields_recorded") is not True):
                R.append("attention_group_scope_unsupported")
            if not _shape(proof.get("configured_group_ids"), [gid]) or not _shape(proof.get("expected_group_ids"), [gid]):
                R.append("group_identity_scope_unverified")
            if (not coord or type(g.get("sent_start")) is not int or g["sent_start"] != 0
                    or type(g.get("sent_block_size")) is not int or g["sent_block_size"] != bs
                    or type(g.get("sent_count")) is not int or g["sent_count"] != full
                    or g.get("sent_dtype") != "uint64" or not _shape(g.get("sent_shape"), [full])
                    or not _int(nt, 1) or count != full - g["start"]):
                R.append("full_load_block_scope_unverified")
            reps = g.get("consumer_reports")
            if type(reps) is not list or len(reps) != 1 or type(reps[0]) is not dict:
                R.append("consumer_worker_scope_unverified")
            else:
                r = reps[0]
                if (any(type(r.get(k)) is not int or r[k] != 0 for k in ("pp_rank", "tp_rank", "record_pp_rank",
                                                                          "record_tp_rank"))
                        or type(r.get("group_start")) is not int or r["group_start"] != g.get("start")
                        or not _shape(r.get("value_shape"), [count, 1]) or r.get("value_dtype") != "uint64"
                        or not (type(r.get("replica_keys")) is list and len(r["replica_keys"]) == 1
                                and _shape(r["replica_keys"][0], [1, 0]))
                        or r.get("skipped") is not False):
                    R.append("consumer_replica_scope_unverified")
                if (not _u64(g.get("sent_fingerprint")) or not _u64(r.get("fingerprint"))
                        or g.get("sent_fingerprint") != r.get("fingerprint")):
                    R.append("group_fingerprint_scope_unverified")
            outcome = g.get("native_group_result")
            wit = rec.get("groups")
            match = ([w for w in wit if type(w) is dict and type(w.get("group_id")) is int and w["group_id"] == gid]
                     if type(wit) is list and len(wit) <= MAX_GROUPS else [])
            if (len(match) != 1 or len(wit) != 1 or not _prim_same(match[0].get("returned_positions"), outcome)
                    or match[0].get("reason") != g.get("native_group_error")):
                R.append("native_group_witness_inconsistent")
            elif ((outcome is None and match[0].get("native_result") not in ("unverified", "not_compared"))
                  or (type(outcome) is list and match[0].get("native_result") != ("mismatch" if outcome else "passed"))):
                R.append("native_group_witness_inconsistent")
            if g.get("compare_called") is not True:
                R.append("group_comparison_not_called")
            elif outcome is None:
                R.append("native_group_not_compared")
                if (native is False and proof.get("source_supported") is True and proof.get("metadata_stable") is True
                        and path == CALL_PATH and _int(rec.get("origin_update_sequence"), 1)
                        and _int(proof.get("plan_sequence"), 1) and g.get("native_group_error") is None
                        and "native_group_witness_inconsistent" not in R and len(match) == 1
                        and match[0].get("native_result") == "not_compared"):
                    compared, established = [], True
            elif (type(outcome) is not list or len(outcome) > count or not _int(g.get("start"))
                  or any(not _int(x) or not g["start"] <= x < g["start"] + count for x in outcome)
                  or len(set(outcome)) != len(outcome)):
                R.append("native_group_result_unverified")
            elif not R:
                compared = list(expected[g["start"]:])
                established = True
            if type(outcome) is list:
                if (native is True and outcome) or (native is False and not outcome and not rec.get("unverified_reasons")):
                    R.append("native_aggregate_group_disagrees")
                    compared, established = None, False
                if (native is False and outcome and "native_group_result_unverified" not in R
                        and "native_group_witness_inconsistent" not in R):
                    res["native_result"] = "mismatch"
    if not expected:
        expected = None
    if native is None:
        R.append("native_verification_not_completed")
    if rec.get("recording_complete") is not True:
        R.append("recording_budget_exhausted" if rec.get("recording_issue") == "global_budget_exhausted"
                 else "recording_scope_incomplete")
    transfer_ok = established and expected is not None and not R
    if transfer_ok:
        res["token_coverage"] = {"prompt_tokens": nt, "transferred_tokens_checked": nt - local,
                                 "decode_cached_tokens_unchecked": local}
        if local:
            R.append(CACHED_PREFIX_REASON)
    missing = sorted(set(expected) - set(compared)) if expected is not None and established else None
    R = list(dict.fromkeys(_gap_reasons(rec, proof) + R))
    complete = not R and bool(expected) and established and compared == expected
    if complete:
        cov = "complete"
    elif transfer_ok and local:
        cov = "partial"
    elif expected is not None and not compared and R == ["native_group_not_compared"]:
        cov = "not_covered"
    else:
        cov = "unknown"
    res.update(expected_units=expected, compared_units=compared if established else None, missing_units=missing,
               coverage=cov, reason="complete_native_checksum_chunk_comparison" if complete else
               (R[0] if R else "scope_metadata_unverified"), reasons=R)
    return res


# ------------------------------------------------------------------------------------------ snapshot report
def _planned_scope_matches(plan: dict, proof: dict) -> bool:
    lp = plan.get("load_plan")
    keys = ("parallel", "speculative_disabled", "native_tp_size", "num_workers", "num_local_computed_tokens",
            "plan_sequence", "num_tokens", "planned_group_count", "configured_group_count", "configured_group_ids")
    if type(lp) is not dict or lp.get("source_supported") is not True or any(
            k not in lp or k not in proof or not ev.same(lp[k], proof[k]) for k in keys):
        return False
    gkeys = ("group_id", "spec_type", "spec_source_supported", "block_size", "sliding_window", "attention_chunk_size",
             "non_causal", "spec_fields_recorded", "start", "block_count")
    a, b = lp.get("groups"), proof.get("groups")
    if type(a) is not list or type(b) is not list or len(a) != len(b):
        return False
    return all(type(x) is dict and type(y) is dict and all(k in x and k in y and ev.same(x[k], y[k]) for k in gkeys)
               for x, y in zip(a, b))


def _count(v) -> bool:
    return type(v) is int and v >= 0


def snapshot_report(snapshot, revision=None) -> dict:
    """Verification calls of one observer snapshot with re-derived scope, plus the snapshot's recording issues
    and observations that have no verification (planned but never compared)."""
    value = snapshot
    if type(value) is not dict or value.get("schema") != SCHEMA:
        raise ev.EvidenceError("unsupported checksum observer snapshot")
    records = value.get("records")
    if type(records) is not list or len(records) > MAX_RECORDS:
        raise ev.EvidenceError("checksum snapshot records exceed the supported bound")
    issues: list[str] = []
    if value.get("profile") != profiles.OBSERVER_PROFILE:
        issues.append("unsupported_source_profile")
    qual = value.get("qualification")
    if qual not in ("cpu_source_functions", "source_bound_candidate"):
        issues.append("source_qualification_unknown")
    if value.get("runtime_qualified") is not False or value.get("release_qualifying") is not False:
        issues.append("unsupported_runtime_or_release_claim")
    source = value.get("source")
    observed = source.get("revision") if type(source) is dict else None
    sel = revision if revision is not None else observed
    if not profiles.supported(sel):
        issues.append("unsupported_source_revision")
        sel = profiles.BASELINE
    prof = profiles.observer_source(sel)
    if (type(source) is not dict or source.get("supported") is not True or source.get("revision") != prof["revision"]
            or not ev.same(source.get("files"), prof["files"])):
        issues.append("declared_source_identity_unverified")
    if value.get("closed") is not True:
        issues.append("observer_not_closed")
    health = value.get("health")
    if (type(health) is not dict or health.get("complete") is not True or health.get("budget_exhausted") is not False
            or any(not _count(health.get(k)) or health[k] != 0 for k in (
                "errors", "dropped_records", "late_calls", "active_calls", "inflight_position_units",
                "inflight_position_bytes"))):
        issues.append("recording_health_unverified")
    b = value.get("budgets")
    keys = ("max_records", "max_units", "max_bytes", "retained_records", "retained_units", "retained_bytes",
            "fixed_metadata_bytes", "reserved_record_bytes", "reserved_state_bytes")
    if (type(b) is not dict or any(not _count(b.get(k)) for k in keys) or not 1 <= b["max_records"] <= MAX_RECORDS
            or not 1 <= b["max_units"] <= MAX_UNITS or not 65536 <= b["max_bytes"] <= 8 * 1024 * 1024):
        raise ev.EvidenceError("unsupported checksum snapshot budgets")
    unit_limit = b["max_units"]
    if (b["retained_records"] != len(records) or len(records) > b["max_records"] or b["retained_units"] > unit_limit
            or b["fixed_metadata_bytes"] != FIXED_METADATA_BYTES or b["reserved_record_bytes"] < b["retained_bytes"]
            or b["fixed_metadata_bytes"] + b["reserved_record_bytes"] + b["reserved_state_bytes"] > b["max_bytes"]):
        issues.append("snapshot_budget_counters_disagree")
    if value.get("closed") is True and (type(b.get("reserved_state_bytes")) is not int or b["reserved_state_bytes"] != 0):
        issues.append("observer_state_not_settled")
    if type(health) is dict and health.get("complete") is True:
        enc = sum(len(json.dumps(r, sort_keys=True, allow_nan=False).encode()) for r in records)
        if enc != b["retained_bytes"]:
            issues.append("snapshot_record_byte_count_disagrees")
    seqs, plans = [], {}
    for r in records:
        if type(r) is not dict or type(r.get("kind")) is not str or not _count(r.get("sequence")) or r["sequence"] == 0:
            issues.append("record_shape_unverified")
            continue
        seqs.append(r["sequence"])
        if r["kind"] not in ("recv_plan", "verification", "not_verified"):
            issues.append("unsupported_record_kind")
        if r["kind"] == "recv_plan" and "plan_sequence" in r:
            p = r["plan_sequence"]
            if not _count(p) or p == 0 or p >= r["sequence"]:
                issues.append("receive_plan_sequence_unverified")
            elif p in plans:
                issues.append("ambiguous_receive_plan")
            else:
                plans[p] = r
    if len(set(seqs)) != len(seqs):
        issues.append("ambiguous_record_sequence")
    if seqs != sorted(seqs):
        issues.append("record_order_unverified")
    issues = list(dict.fromkeys(issues))
    rows, total, joined = [], 0, set()
    for i, r in enumerate(records):
        if type(r) is not dict or r.get("kind") != "verification":
            continue
        try:
            d = classify_verification(r, max_units=unit_limit)
        except (TypeError, ValueError, KeyError, IndexError) as e:
            raise ev.EvidenceError("unsupported verification metadata: " + str(e)) from e
        reasons = list(issues)
        req = r.get("request_id")
        if type(req) is not str or not req or len(req) > 1024:
            reasons.append("request_identity_unverified")
            req = None
        proof = r.get("proof") if type(r.get("proof")) is dict else {}
        pid = proof.get("plan_sequence")
        plan = plans.get(pid) if _count(pid) else None
        upd, seq = r.get("origin_update_sequence"), r.get("sequence")
        if (plan is None or plan.get("request_id") != req or not _count(upd) or not _count(seq)
                or not plan["sequence"] < upd < seq):
            reasons.append("receive_plan_to_verification_join_unverified")
        elif pid in joined:
            reasons.append("ambiguous_receive_plan_verification")
        else:
            joined.add(pid)
            if not _planned_scope_matches(plan, proof):
                reasons.append("planned_chunk_scope_disagrees_with_verification")
        for name, want in d.items():
            if name in r and not ev.same(r[name], want):
                reasons.append("derived_observation_disagrees:" + name)
        total += len(d.get("expected_units") or []) + len(d.get("compared_units") or [])
        if total > unit_limit:
            raise ev.EvidenceError("aggregate checksum chunk scope exceeds its bound")
        row = {"record_index": i, "sequence": r.get("sequence"), "request_id": req, "native_result": d["native_result"],
               "native_return": d["native_return"], "conditional_scope": d,
               "coverage": "unknown" if reasons else d["coverage"], "reason": reasons[0] if reasons else d["reason"],
               "recording_issues": list(dict.fromkeys(reasons))}
        row["engine_pass_not_covered_reason"] = next(
            (n for n in (CACHED_PREFIX_REASON, "partial_checksum_span", "empty_replica_inputs")
             if d["native_result"] == "passed" and n in d["reasons"]), None)
        rows.append(row)
    retained, shapes_ok = 0, True
    for r in records:
        if type(r) is not dict:
            continue
        for k in ("expected_units", "compared_units", "missing_units"):
            u = r.get(k)
            if u is None:
                continue
            if type(u) is not list or any(type(x) is not str for x in u):
                shapes_ok = False
            else:
                retained += len(u)
    if not shapes_ok or retained != b["retained_units"]:
        issues.append("snapshot_retained_units_disagree")
        for row in rows:
            row.update(coverage="unknown", reason="snapshot_retained_units_disagree")
            row["recording_issues"].append("snapshot_retained_units_disagree")
    unverified = []
    for i, r in enumerate(records):
        if type(r) is not dict:
            continue
        p = r.get("plan_sequence")
        if r.get("kind") == "not_verified" or (r.get("kind") == "recv_plan" and (not _count(p) or p not in joined)):
            scheduled = r.get("kind") == "recv_plan" and _count(p)
            unverified.append({"record_index": i, "sequence": r.get("sequence"), "request_id": r.get("request_id"),
                               "reason": "receive_plan_without_verification" if scheduled
                               else r.get("reason", "native_verification_not_recorded"),
                               "native_plan_reason": r.get("reason") if scheduled else None, "coverage": "unknown"})
    if not rows:
        issues.append("no_recorded_native_verification_calls")
    return {"qualification": qual, "verification_calls": rows, "unverified_observations": unverified,
            "hold_reasons": list(dict.fromkeys(issues + ["runtime_qualification_pending",
                                                         "independent_client_inventory_not_joined",
                                                         "joint_release_profile_not_qualified"])),
            "summary": {"recorded_events": len(records), "verification_calls": len(rows),
                        "native_results": dict(Counter(r["native_result"] for r in rows)),
                        "chunk_scope": dict(Counter(r["coverage"] for r in rows))}}


# ------------------------------------------------------------------------------------------ cache accounting
def cache_snapshot(snapshot, context: dict, role: str, revision: str) -> tuple[list, list]:
    """Validated prefill-accounting records of one engine; missing data is never read as zero."""
    if (type(snapshot) is not dict or snapshot.get("schema") != CACHE_SCHEMA or snapshot.get("role") != role
            or snapshot.get("closed") is not True or not _int(snapshot.get("process_id"), 1)
            or snapshot.get("qualification") not in ("source_bound_candidate", "cpu_source_functions")
            or any(snapshot.get(k) != v for k, v in context.items())
            or type(snapshot.get("source")) is not dict or snapshot["source"].get("supported") is not True
            or snapshot.get("source") != dict(profiles.cache_source(revision), supported=True)):
        return [], ["native_cache_accounting_identity_unverified"]
    R = []
    health, lim, records = snapshot.get("health"), snapshot.get("budgets"), snapshot.get("records")
    if (type(health) is not dict or health.get("complete") is not True or health.get("budget_exhausted") is not False
            or any(type(health.get(k)) is not int or health[k] != 0 for k in ("errors", "dropped_records",
                                                                             "late_calls", "active_calls"))):
        R.append("native_cache_accounting_incomplete")
    if type(records) is not list or len(records) > CACHE_MAX_RECORDS:
        return [], R + ["native_cache_accounting_records_unverified"]
    if (type(lim) is not dict or not _int(lim.get("max_records"), 1, CACHE_MAX_RECORDS)
            or not _int(lim.get("max_bytes"), 65536, CACHE_MAX_BYTES)
            or type(lim.get("retained_records")) is not int or lim["retained_records"] != len(records)
            or type(lim.get("retained_bytes")) is not int
            or lim["retained_bytes"] != sum(len(ev.json_bytes(r)) for r in records)
            or type(lim.get("fixed_bytes")) is not int or lim["fixed_bytes"] != CACHE_FIXED_BYTES
            or len(records) > lim["max_records"] or lim["retained_bytes"] + CACHE_FIXED_BYTES > lim["max_bytes"]):
        R.append("native_cache_accounting_budget_unverified")
    seq = [r.get("sequence") if type(r) is dict else None for r in records]
    if any(not _int(s, 1) for s in seq) or seq != list(range(1, len(seq) + 1)):
        R.append("native_cache_accounting_sequence_unverified")
    for row in records:
        if (type(row) is not dict or not _text(row.get("request_id")) or not _int(row.get("output_tokens"), 0, MAX_PROMPT_TOKENS)
                or not _int(row.get("preemptions"), 0, MAX_PROMPT_TOKENS) or row.get("status") not in CACHE_STATUSES
                or "stats" not in row):
            R.append("native_cache_accounting_record_unverified")
            continue
        v = row["stats"]
        if v is not None and (type(v) is not dict or set(v) != set(CACHE_FIELDS)
                              or any(not _int(v[k], 0, MAX_PROMPT_TOKENS) for k in CACHE_FIELDS)
                              or not _int(row.get("prompt_tokens"), 1, MAX_PROMPT_TOKENS)
                              or v["num_prompt_tokens"] != row["prompt_tokens"]
                              or v["num_cached_tokens"] != v["num_local_cached_tokens"] + v["num_external_cached_tokens"]
                              or v["num_prompt_tokens"] != v["num_computed_tokens"] + v["num_cached_tokens"]):
            R.append("native_cache_accounting_counts_unverified")
    return records, list(dict.fromkeys(R))


def request_usage(records: list, internal_id, prompt_tokens, prompt_sha256, completion_tokens):
    """(first stats, reasons) of one request: exactly one record with stats, monotone output counts ending at the
    client's completion count, a clean finish, and no preemption."""
    sel = [r for r in records if type(r) is dict and r.get("request_id") == internal_id]
    initial = [r for r in sel if r.get("stats") is not None]
    if len(initial) != 1 or not sel:
        return None, ["unambiguous_native_prefill_stats_missing"]
    first, last = initial[0], sel[-1]
    R = []
    if first.get("prompt_tokens") != prompt_tokens or first.get("prompt_sha256") != prompt_sha256 or first is not sel[0]:
        R.append("native_cache_prompt_binding_unverified")
    counts = [r.get("output_tokens") for r in sel]
    if (any(not _int(n) for n in counts) or counts != sorted(counts) or not _int(completion_tokens, 1)
            or counts[-1] != completion_tokens or last.get("status") not in FINISHED_OK
            or any(r.get("status") != "RUNNING" for r in sel[:-1])):
        R.append("native_cache_terminal_request_unverified")
    if any(type(r.get("preemptions")) is not int or r["preemptions"] != 0 for r in sel):
        R.append("native_cache_preempted_request_unsupported")
    return (first.get("stats") if not R else None), R
