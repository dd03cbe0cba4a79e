"""Offline interpretation of recorded KV-checksum observations, as ordered tables of findings.

A recording holds, per decode engine, a closed snapshot (`sdcguard.checksum-observer.v1`) of two record kinds:
`recv_plan` (what the consumer planned to receive and compare: token count, locally cached prefix, block groups,
the producer's checksum array shape and fingerprint) and `verification` (the native comparison call: its return,
per-group witnesses, and the proof of scope). From these the gate re-derives, never trusting a stored verdict:

    expected units   group:G:chunk:i  for every 16-token chunk of the prompt
    compared units   the chunks from the first transferred chunk on, when the comparison is established
    coverage         complete | partial (cached prefix not compared) | not_covered | unknown
    token coverage   prompt tokens, transferred tokens checked, decode-cache tokens reused unchecked

and the prefill-accounting snapshot (`sdcguard.native-prefill-accounting.v1`) gives per-request cache counts.

How it is organised. Every defect a record can have is one `Finding`: the reason string the verdict carries and
a predicate over a read-only view of the record (`_Call`, `_Snapshot`, `_CacheSnapshot`). Findings are grouped in
tables by the part of the record they need (the whole call, its single block group once that group's shape is
sound, the group's comparison outcome, the recording's completeness), and a record's reasons are the findings
that hold, in table order. What a verdict derives beyond its reasons (the compared units, the token coverage,
the coverage word) is computed from the view and the findings after the tables ran.

The reason strings, their order and the derived fields are the recorded-evidence contract of the reference's
recorder (src/sdcguard/kv_checksum_observer.py:84-330, checksum_observer_report.py:70-246,
prefix_cache_observer.py:246-313): the same recordings must get the same verdicts. This package's own P/D engine
writes records of the same schema (sdcguard_b200.serve.pd).
"""
from __future__ import annotations

import json
from collections import Counter
from typing import Callable, NamedTuple, Optional

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
RANKS_OF_ONE_WORKER = ("pp_rank", "tp_rank", "record_pp_rank", "record_tp_rank")
PARALLEL_AXES = ("tp", "pp", "dp", "dcp", "pcp")
# the fixed hold reasons of every observer report: what an offline reading of one snapshot can never establish
REPORT_LIMITS = ("runtime_qualification_pending", "independent_client_inventory_not_joined",
                 "joint_release_profile_not_qualified")
# a passing native call can still leave chunks uncompared; the first of these reasons names why
ENGINE_PASS_GAPS = (CACHED_PREFIX_REASON, "partial_checksum_span", "empty_replica_inputs")


# ------------------------------------------------------------------------------------------ value predicates
def _int(v, lo=0, hi=2 ** 63 - 1) -> bool:
    """An exact int (not bool) in [lo, hi]."""
    return type(v) is int and lo <= v <= hi


def _u64(v) -> bool:
    return type(v) is int and 0 <= v < 2 ** 64


def _text(v, n=1024) -> bool:
    return type(v) is str and 0 < len(v) <= n and "\x00" not in v


def _ints_equal(v, want: list) -> bool:
    """A list of exact ints equal to `want` element by element (a shape or an id list)."""
    return type(v) is list and len(v) == len(want) and all(type(x) is int and x == y for x, y in zip(v, want))


def _one_dict(v) -> Optional[dict]:
    """The only element of a one-element list of objects, else None."""
    return v[0] if type(v) is list and len(v) == 1 and type(v[0]) is dict else None


def _canon(v) -> Optional[str]:
    try:
        return json.dumps(v, sort_keys=True, allow_nan=False)
    except (ValueError, TypeError):
        return None


def _same_plain(a, b) -> bool:
    ca, cb = _canon(a), _canon(b)
    return ca is not None and ca == cb


def _dedup(xs) -> list:
    return list(dict.fromkeys(xs))


class Finding(NamedTuple):
    reason: str
    holds: Callable[..., bool]


def _run(table, view) -> list[str]:
    return [f.reason for f in table if f.holds(view)]


# ------------------------------------------------------------------------------------------ one verification call
class _Call:
    """Read-only view of one `verification` record with every field a finding needs, typed or None."""

    def __init__(self, record, max_units: int):
        self.rec = rec = record if type(record) is dict else {}
        self.max_units = max_units
        self.native = rec.get("native_return") if type(rec.get("native_return")) is bool else None
        self.proof = proof = rec.get("proof") if type(rec.get("proof")) is dict else {}
        self.groups = proof.get("groups") if type(proof.get("groups")) is list else []
        self.unv = rec.get("unverified_reasons", [])
        self.local = proof.get("num_local_computed_tokens")
        self.nt = proof.get("num_tokens")
        self.et = proof.get("expected_num_tokens")
        self.path_ok = (proof.get("call_path") == CALL_PATH and _int(rec.get("origin_update_sequence"), 1)
                        and _int(proof.get("plan_sequence"), 1))
        # the one block group, when the proof lists exactly one object
        self.g = g = self.groups[0] if len(self.groups) == 1 and type(self.groups[0]) is dict else None
        self.gid = g.get("group_id") if g else None
        self.bs = g.get("block_size") if g else None
        self.count = g.get("block_count") if g else None
        self.shape_ok = g is not None and not (proof.get("scope_budget_refused") is True or not _int(self.gid)
                                               or not _int(self.bs, 1) or not _int(self.count, 1)
                                               or self.count > max_units // 2)
        self.full = (self.nt + self.bs - 1) // self.bs if self.shape_ok and _int(self.nt, 1) else None
        self.report = _one_dict(g.get("consumer_reports")) if g else None
        self.outcome = g.get("native_group_result") if g else None
        wit = rec.get("groups")
        self.wit = wit
        self.match = ([w for w in wit if type(w) is dict and type(w.get("group_id")) is int and w["group_id"] == self.gid]
                      if g and type(wit) is list and len(wit) <= MAX_GROUPS else [])

    # -- derived facts the tables share
    def unv_shape_ok(self) -> bool:
        u = self.unv
        return type(u) is list and len(u) <= MAX_GROUPS and all(type(x) is str and len(x) <= 512 for x in u)

    def coordinates_ok(self) -> bool:
        """The group's chunk coordinates are those of a full-attention load after a 16-aligned local prefix."""
        g, bs, local, nt = self.g, self.bs, self.local, self.nt
        return (g.get("spec_type") == "FullAttentionSpec" and g.get("spec_source_supported") is True
                and _int(local) and _int(nt, 1) and local < nt and local % bs == 0
                and type(g.get("start")) is int and g["start"] == local // bs
                and type(g.get("sent_block_size")) is int and g["sent_block_size"] == bs
                and self.full <= self.max_units // 2)

    def expected(self) -> Optional[list]:
        if self.shape_ok and self.coordinates_ok():
            return [f"group:{self.gid}:chunk:{i}" for i in range(self.full)]
        return None

    def full_load_ok(self) -> bool:
        g = self.g
        return (self.coordinates_ok() and g.get("sent_start") == 0 and type(g.get("sent_start")) is int
                and type(g.get("sent_block_size")) is int and g["sent_block_size"] == self.bs
                and type(g.get("sent_count")) is int and g["sent_count"] == self.full
                and g.get("sent_dtype") == "uint64" and _ints_equal(g.get("sent_shape"), [self.full])
                and _int(self.nt, 1) and self.count == self.full - g["start"])

    def replica_ok(self) -> bool:
        r, g = self.report, self.g
        keys = r.get("replica_keys")
        return (all(type(r.get(k)) is int and r[k] == 0 for k in RANKS_OF_ONE_WORKER)
                and type(r.get("group_start")) is int and r["group_start"] == g.get("start")
                and _ints_equal(r.get("value_shape"), [self.count, 1]) and r.get("value_dtype") == "uint64"
                and type(keys) is list and len(keys) == 1 and _ints_equal(keys[0], [1, 0])
                and r.get("skipped") is False)

    def fingerprints_agree(self) -> bool:
        a, b = self.g.get("sent_fingerprint"), self.report.get("fingerprint")
        return _u64(a) and _u64(b) and a == b

    def witness_consistent(self) -> bool:
        """The per-group witness of the call agrees with the group's recorded outcome."""
        m, wit, outcome = self.match, self.wit, self.outcome
        if len(m) != 1 or len(wit) != 1 or not _same_plain(m[0].get("returned_positions"), outcome) \
                or m[0].get("reason") != self.g.get("native_group_error"):
            return False
        said = m[0].get("native_result")
        if outcome is None:
            return said in ("unverified", "not_compared")
        if type(outcome) is list:
            return said == ("mismatch" if outcome else "passed")
        return True

    def outcome_kind(self) -> str:
        """not_called | none (called, no result) | invalid (a result that is not a set of in-range positions) |
        listed (the mismatching positions, possibly none)."""
        g, out = self.g, self.outcome
        if g.get("compare_called") is not True:
            return "not_called"
        if out is None:
            return "none"
        start = g.get("start")
        if (type(out) is not list or len(out) > self.count or not _int(start)
                or any(not _int(x) or not start <= x < start + self.count for x in out) or len(set(out)) != len(out)):
            return "invalid"
        return "listed"

    def aggregate_disagrees(self) -> bool:
        out = self.outcome
        return type(out) is list and ((self.native is True and bool(out))
                                      or (self.native is False and not out and not self.rec.get("unverified_reasons")))


_CALL_TABLE = (
    Finding("scope_budget_refused", lambda c: c.proof.get("scope_budget_refused") is True),
    Finding("native_unverified_reason_shape_invalid", lambda c: not c.unv_shape_ok()),
    Finding("native_comparison_unverified", lambda c: c.unv_shape_ok() and bool(c.unv)),
    Finding("native_engine_exception_present", lambda c: c.rec.get("engine_exception") is not None),
    Finding("native_call_path_unverified", lambda c: not c.path_ok),
    Finding("source_profile_unverified", lambda c: c.proof.get("source_supported") is not True),
    Finding("scope_metadata_changed_or_unobserved", lambda c: c.proof.get("metadata_stable") is not True),
    Finding("parallel_scope_unsupported", lambda c: not (
        type(c.proof.get("parallel")) is dict and all(_int(c.proof["parallel"].get(k), 1) and c.proof["parallel"][k] == 1
                                                      for k in PARALLEL_AXES)
        and type(c.proof.get("num_workers")) is int and c.proof["num_workers"] == 1
        and type(c.proof.get("native_tp_size")) is int and c.proof["native_tp_size"] == 1)),
    Finding("speculative_configuration_unknown_or_enabled", lambda c: c.proof.get("speculative_disabled") is not True),
    Finding("producer_checksum_payload_missing_or_unverified",
            lambda c: c.proof.get("producer_payload_present") is not True),
    Finding("local_prefix_scope_unsupported", lambda c: not (_int(c.local) and _int(c.nt, 1) and c.local < c.nt)),
    Finding("producer_consumer_token_scope_differs",
            lambda c: not (_int(c.nt, 1) and type(c.et) is int and c.nt == c.et)),
    Finding("group_scope_unsupported", lambda c: not (
        all(type(c.proof.get(k)) is int and c.proof[k] == 1
            for k in ("expected_tp_size", "planned_group_count", "configured_group_count"))
        and len(c.groups) == 1)),
    Finding("worker_rank_scope_unverified", lambda c: not (
        type(c.proof.get("worker_ranks")) is list and len(c.proof["worker_ranks"]) == 1
        and _ints_equal(c.proof["worker_ranks"][0], [0, 0])
        and type(c.proof.get("worker_report_count")) is int and c.proof["worker_report_count"] == 1)),
)

# the single block group, once its id, block size and count are sound
_GROUP_TABLE = (
    Finding("local_prefix_coordinate_scope_unverified", lambda c: not c.coordinates_ok()),
    Finding("attention_group_scope_unsupported", lambda c: not (
        c.g.get("spec_type") == "FullAttentionSpec" and c.g.get("spec_source_supported") is True
        and c.g.get("sliding_window") is None and c.g.get("attention_chunk_size") is None
        and c.g.get("non_causal") is False and c.g.get("spec_fields_recorded") is True)),
    Finding("group_identity_scope_unverified", lambda c: not (
        _ints_equal(c.proof.get("configured_group_ids"), [c.gid])
        and _ints_equal(c.proof.get("expected_group_ids"), [c.gid]))),
    Finding("full_load_block_scope_unverified", lambda c: not c.full_load_ok()),
    Finding("consumer_worker_scope_unverified", lambda c: c.report is None),
    Finding("consumer_replica_scope_unverified", lambda c: c.report is not None and not c.replica_ok()),
    Finding("group_fingerprint_scope_unverified", lambda c: c.report is not None and not c.fingerprints_agree()),
    Finding("native_group_witness_inconsistent", lambda c: not c.witness_consistent()),
)

_OUTCOME_TABLE = (
    Finding("group_comparison_not_called", lambda c: c.outcome_kind() == "not_called"),
    Finding("native_group_not_compared", lambda c: c.outcome_kind() == "none"),
    Finding("native_group_result_unverified", lambda c: c.outcome_kind() == "invalid"),
)

_COMPLETION_TABLE = (
    Finding("native_verification_not_completed", lambda c: c.native is None),
    Finding("recording_budget_exhausted", lambda c: c.rec.get("recording_complete") is not True
            and c.rec.get("recording_issue") == "global_budget_exhausted"),
    Finding("recording_scope_incomplete", lambda c: c.rec.get("recording_complete") is not True
            and c.rec.get("recording_issue") != "global_budget_exhausted"),
)


def _engine_pass_gaps(c: _Call) -> list[str]:
    """A native pass of one group that still leaves chunks uncompared: the consumer had no replica inputs to
    compare, or the compared span does not line up with the producer's span (or a last chunk holds different
    token counts on the two sides)."""
    proof, rec = c.proof, c.rec
    g, w = _one_dict(proof.get("groups")), _one_dict(rec.get("groups"))
    clean_pass = (rec.get("native_return") is True and proof.get("source_supported") is True
                  and proof.get("metadata_stable") is True and rec.get("engine_exception") is None
                  and rec.get("unverified_reasons") == [] and g is not None and w is not None
                  and g.get("compare_called") is True and g.get("native_group_result") == []
                  and g.get("native_group_error") is None and w.get("native_result") == "passed"
                  and w.get("returned_positions") == [] and w.get("reason") is None and _int(g.get("group_id"))
                  and type(w.get("group_id")) is int and w["group_id"] == g["group_id"])
    if not clean_pass:
        return []
    gaps = []
    count, rep = g.get("block_count"), _one_dict(g.get("consumer_reports"))
    if (_int(count, 1) and rep is not None and type(rep.get("replica_keys")) is list and rep["replica_keys"] == []
            and _ints_equal(rep.get("value_shape"), [count, 0])):
        gaps.append("empty_replica_inputs")
    bs, start, scount, sstart = g.get("block_size"), g.get("start"), g.get("sent_count"), g.get("sent_start")
    nt, et = proof.get("num_tokens"), proof.get("expected_num_tokens")
    geometry = (g.get("spec_type") == "FullAttentionSpec" and g.get("spec_source_supported") is True
                and _int(bs, 1) and type(g.get("sent_block_size")) is int and bs == g["sent_block_size"]
                and _int(start) and _int(sstart) and _int(count, 1) and _int(scount, 1) and _int(nt, 1) and _int(et, 1)
                and count == -(-nt // bs) - start and scount == -(-et // bs) - sstart
                and _ints_equal(g.get("sent_shape"), [scount]))
    if not geometry:
        return gaps
    lo, hi = max(start, sstart), min(start + count, sstart + scount)
    if lo >= hi:
        return gaps
    uneven = lo > start or hi < start + count

    def tokens_in(chunk, total):
        return min(bs, max(0, total - chunk * bs))
    last_chunks = {(nt - 1) // bs, (et - 1) // bs}
    if uneven or any(lo <= pos < hi and tokens_in(pos, nt) != tokens_in(pos, et) for pos in last_chunks):
        gaps.append("partial_checksum_span")
    return gaps


def classify_verification(record, *, max_units: int = MAX_UNITS) -> dict:
    """Re-derive the conditional chunk scope of one `verification` record from its primitive observations."""
    if not _int(max_units, 1) or max_units > 1048576:
        raise ValueError("max_units must be between 1 and 1048576")
    c = _Call(record, max_units)
    reasons = _run(_CALL_TABLE, c)
    expected = compared = None
    established = False
    mismatch = False
    if c.g is not None:
        if not c.shape_ok:
            reasons.append("chunk_scope_budget_or_shape_invalid")
        else:
            expected = c.expected()
            reasons += _run(_GROUP_TABLE, c)
            before_outcome = bool(reasons)
            reasons += _run(_OUTCOME_TABLE, c)
            kind = c.outcome_kind()
            if kind == "none":
                # a native "not compared" answer that the whole call path vouches for: established, nothing compared
                vouched = (c.native is False and c.proof.get("source_supported") is True
                           and c.proof.get("metadata_stable") is True and c.path_ok
                           and c.g.get("native_group_error") is None and c.witness_consistent()
                           and len(c.match) == 1 and c.match[0].get("native_result") == "not_compared")
                if vouched:
                    compared, established = [], True
            elif kind == "listed" and not before_outcome:
                compared, established = list(expected[c.g["start"]:]), True
            if c.aggregate_disagrees():
                reasons.append("native_aggregate_group_disagrees")
                compared, established = None, False
            mismatch = (c.native is False and type(c.outcome) is list and bool(c.outcome)
                        and kind != "invalid" and c.witness_consistent())
    reasons += _run(_COMPLETION_TABLE, c)
    token_cov = {"prompt_tokens": None, "transferred_tokens_checked": None, "decode_cached_tokens_unchecked": None}
    transfer_ok = established and expected is not None and not reasons
    if transfer_ok:
        token_cov = {"prompt_tokens": c.nt, "transferred_tokens_checked": c.nt - c.local,
                     "decode_cached_tokens_unchecked": c.local}
        if c.local:
            reasons.append(CACHED_PREFIX_REASON)
    missing = sorted(set(expected) - set(compared)) if expected is not None and established else None
    reasons = _dedup(_engine_pass_gaps(c) + reasons)
    complete = not reasons and bool(expected) and established and compared == expected
    if complete:
        coverage = "complete"
    elif transfer_ok and c.local:
        coverage = "partial"
    elif expected is not None and not compared and reasons == ["native_group_not_compared"]:
        coverage = "not_covered"
    else:
        coverage = "unknown"
    return {"native_return": c.native,
            "native_result": "mismatch" if mismatch else "passed" if c.native is True else "unverified",
            "expected_units": expected, "compared_units": compared if established else None,
            "missing_units": missing, "coverage": coverage,
            "reason": "complete_native_checksum_chunk_comparison" if complete else
            (reasons[0] if reasons else "scope_metadata_unverified"),
            "reasons": reasons, "token_coverage": token_cov}


# ------------------------------------------------------------------------------------------ snapshot report
PLAN_KEYS = ("parallel", "speculative_disabled", "native_tp_size", "num_workers", "num_local_computed_tokens",
             "plan_sequence", "num_tokens", "planned_group_count", "configured_group_count", "configured_group_ids")
PLAN_GROUP_KEYS = ("group_id", "spec_type", "spec_source_supported", "block_size", "sliding_window",
                   "attention_chunk_size", "non_causal", "spec_fields_recorded", "start", "block_count")


def plan_matches_proof(plan: dict, proof: dict) -> bool:
    """The receive plan's load scope is the scope the verification's proof states, key for key and group for
    group (the comparison checked what was planned)."""
    lp = plan.get("load_plan")
    if type(lp) is not dict or lp.get("source_supported") is not True:
        return False

    def agree(a: dict, b: dict, keys) -> bool:
        return all(k in a and k in b and ev.same(a[k], b[k]) for k in keys)
    if not agree(lp, proof, PLAN_KEYS):
        return False
    a, b = lp.get("groups"), proof.get("groups")
    if type(a) is not list or type(b) is not list or len(a) != len(b):
        return False
    return all(type(x) is dict and type(y) is dict and agree(x, y, PLAN_GROUP_KEYS) for x, y in zip(a, b))


def _count(v) -> bool:
    return type(v) is int and v >= 0


BUDGET_KEYS = ("max_records", "max_units", "max_bytes", "retained_records", "retained_units", "retained_bytes",
               "fixed_metadata_bytes", "reserved_record_bytes", "reserved_state_bytes")
HEALTH_ZERO = ("errors", "dropped_records", "late_calls", "active_calls", "inflight_position_units",
               "inflight_position_bytes")


class _Snapshot:
    """Read-only view of one observer snapshot (its schema and record list already checked)."""

    def __init__(self, value: dict, revision):
        self.v = value
        self.records = value["records"]
        self.source = value.get("source") if type(value.get("source")) is dict else None
        observed = self.source.get("revision") if self.source else None
        self.revision = revision if revision is not None else observed
        self.health = value.get("health")
        self.b = value.get("budgets")

    def health_ok(self) -> bool:
        h = self.health
        return (type(h) is dict and h.get("complete") is True and h.get("budget_exhausted") is False
                and all(_count(h.get(k)) and h[k] == 0 for k in HEALTH_ZERO))

    def source_identity_ok(self) -> bool:
        pin = profiles.observer_source(self.revision if profiles.supported(self.revision) else profiles.BASELINE)
        s = self.source
        return (s is not None and s.get("supported") is True and s.get("revision") == pin["revision"]
                and ev.same(s.get("files"), pin["files"]))

    def budgets_readable(self) -> bool:
        b = self.b
        return (type(b) is dict and all(_count(b.get(k)) for k in BUDGET_KEYS) and 1 <= b["max_records"] <= MAX_RECORDS
                and 1 <= b["max_units"] <= MAX_UNITS and 65536 <= b["max_bytes"] <= 8 * 1024 * 1024)

    def counters_agree(self) -> bool:
        b, n = self.b, len(self.records)
        return (b["retained_records"] == n and n <= b["max_records"] and b["retained_units"] <= b["max_units"]
                and b["fixed_metadata_bytes"] == FIXED_METADATA_BYTES
                and b["reserved_record_bytes"] >= b["retained_bytes"]
                and b["fixed_metadata_bytes"] + b["reserved_record_bytes"] + b["reserved_state_bytes"] <= b["max_bytes"])

    def encoded_bytes(self) -> int:
        return sum(len(json.dumps(r, sort_keys=True, allow_nan=False).encode()) for r in self.records)


_SNAPSHOT_HEAD = (
    Finding("unsupported_source_profile", lambda s: s.v.get("profile") != profiles.OBSERVER_PROFILE),
    Finding("source_qualification_unknown",
            lambda s: s.v.get("qualification") not in ("cpu_source_functions", "source_bound_candidate")),
    Finding("unsupported_runtime_or_release_claim",
            lambda s: s.v.get("runtime_qualified") is not False or s.v.get("release_qualifying") is not False),
    Finding("unsupported_source_revision", lambda s: not profiles.supported(s.revision)),
    Finding("declared_source_identity_unverified", lambda s: not s.source_identity_ok()),
    Finding("observer_not_closed", lambda s: s.v.get("closed") is not True),
    Finding("recording_health_unverified", lambda s: not s.health_ok()),
)

# after the budgets were found readable
_SNAPSHOT_BUDGET = (
    Finding("snapshot_budget_counters_disagree", lambda s: not s.counters_agree()),
    Finding("observer_state_not_settled", lambda s: s.v.get("closed") is True and s.b["reserved_state_bytes"] != 0),
    Finding("snapshot_record_byte_count_disagrees", lambda s: type(s.health) is dict
            and s.health.get("complete") is True and s.encoded_bytes() != s.b["retained_bytes"]),
)


def _record_findings(records) -> tuple[list[str], dict]:
    """Per-record shape and receive-plan indexing findings, and the receive plans by their plan sequence."""
    out, plans, seqs = [], {}, []
    for r in records:
        if type(r) is not dict or type(r.get("kind")) is not str or not _count(r.get("sequence")) or r["sequence"] == 0:
            out.append("record_shape_unverified")
            continue
        seqs.append(r["sequence"])
        kind = r["kind"]
        if kind not in ("recv_plan", "verification", "not_verified"):
            out.append("unsupported_record_kind")
        if kind != "recv_plan" or "plan_sequence" not in r:
            continue
        p = r["plan_sequence"]
        if not _count(p) or p == 0 or p >= r["sequence"]:
            out.append("receive_plan_sequence_unverified")
        elif p in plans:
            out.append("ambiguous_receive_plan")
        else:
            plans[p] = r
    if len(set(seqs)) != len(seqs):
        out.append("ambiguous_record_sequence")
    if seqs != sorted(seqs):
        out.append("record_order_unverified")
    return out, plans


def _retained_units(records) -> Optional[int]:
    """Units retained by the records' unit lists, or None when a list is malformed."""
    n = 0
    for r in records:
        if type(r) is not dict:
            continue
        for k in ("expected_units", "compared_units", "missing_units"):
            u = r.get(k)
            if u is None:
                continue
            if type(u) is not list or any(type(x) is not str for x in u):
                return None
            n += len(u)
    return n


def snapshot_report(snapshot, revision=None) -> dict:
    """Verification calls of one observer snapshot with re-derived scope, plus the snapshot's recording issues
    and observations that have no verification (planned but never compared)."""
    if type(snapshot) is not dict or snapshot.get("schema") != SCHEMA:
        raise ev.EvidenceError("unsupported checksum observer snapshot")
    records = snapshot.get("records")
    if type(records) is not list or len(records) > MAX_RECORDS:
        raise ev.EvidenceError("checksum snapshot records exceed the supported bound")
    s = _Snapshot(snapshot, revision)
    issues = _run(_SNAPSHOT_HEAD, s)
    if not s.budgets_readable():
        raise ev.EvidenceError("unsupported checksum snapshot budgets")
    issues += _run(_SNAPSHOT_BUDGET, s)
    per_record, plans = _record_findings(records)
    issues = _dedup(issues + per_record)
    unit_limit = s.b["max_units"]
    rows, joined, total = [], set(), 0
    for i, r in enumerate(records):
        if type(r) is not dict or r.get("kind") != "verification":
            continue
        try:
            d = classify_verification(r, max_units=unit_limit)
        except (TypeError, ValueError, KeyError, IndexError) as e:
            raise ev.EvidenceError("unsupported verification metadata: " + str(e)) from e
        row_issues = list(issues)
        req = r.get("request_id")
        if not (type(req) is str and req and len(req) <= 1024):
            row_issues.append("request_identity_unverified")
            req = None
        proof = r.get("proof") if type(r.get("proof")) is dict else {}
        pid = proof.get("plan_sequence")
        plan = plans.get(pid) if _count(pid) else None
        upd, seq = r.get("origin_update_sequence"), r.get("sequence")
        ordered = (plan is not None and plan.get("request_id") == req and _count(upd) and _count(seq)
                   and plan["sequence"] < upd < seq)
        if not ordered:
            row_issues.append("receive_plan_to_verification_join_unverified")
        elif pid in joined:
            row_issues.append("ambiguous_receive_plan_verification")
        else:
            joined.add(pid)
            if not plan_matches_proof(plan, proof):
                row_issues.append("planned_chunk_scope_disagrees_with_verification")
        row_issues += ["derived_observation_disagrees:" + k for k, want in d.items() if k in r and not ev.same(r[k], want)]
        total += len(d.get("expected_units") or []) + len(d.get("compared_units") or [])
        if total > unit_limit:
            raise ev.EvidenceError("aggregate checksum chunk scope exceeds its bound")
        gap = next((n for n in ENGINE_PASS_GAPS if d["native_result"] == "passed" and n in d["reasons"]), None)
        rows.append({"record_index": i, "sequence": r.get("sequence"), "request_id": req,
                     "native_result": d["native_result"], "native_return": d["native_return"],
                     "conditional_scope": d, "coverage": "unknown" if row_issues else d["coverage"],
                     "reason": row_issues[0] if row_issues else d["reason"],
                     "recording_issues": _dedup(row_issues), "engine_pass_not_covered_reason": gap})
    retained = _retained_units(records)
    if retained is None or retained != s.b["retained_units"]:
        issues.append("snapshot_retained_units_disagree")
        for row in rows:
            row.update(coverage="unknown", reason="snapshot_retained_units_disagree")
            row["recording_issues"].append("snapshot_retained_units_disagree")
    unverified = []
    for i, r in enumerate(records):
        if type(r) is not dict:
            continue
        p = r.get("plan_sequence")
        planned_only = r.get("kind") == "recv_plan" and (not _count(p) or p not in joined)
        if r.get("kind") != "not_verified" and not planned_only:
            continue
        scheduled = r.get("kind") == "recv_plan" and _count(p)
        unverified.append({"record_index": i, "sequence": r.get("sequence"), "request_id": r.get("request_id"),
                           "reason": "receive_plan_without_verification" if scheduled
                           else r.get("reason", "native_verification_not_recorded"),
                           "native_plan_reason": r.get("reason") if scheduled else None, "coverage": "unknown"})
    if not rows:
        issues.append("no_recorded_native_verification_calls")
    return {"qualification": snapshot.get("qualification"), "verification_calls": rows,
            "unverified_observations": unverified, "hold_reasons": _dedup(issues + list(REPORT_LIMITS)),
            "summary": {"recorded_events": len(records), "verification_calls": len(rows),
                        "native_results": dict(Counter(r["native_result"] for r in rows)),
                        "chunk_scope": dict(Counter(r["coverage"] for r in rows))}}


# ------------------------------------------------------------------------------------------ cache accounting
class _CacheSnapshot:
    def __init__(self, snap, context: dict, role: str, revision: str):
        self.s, self.context, self.role, self.revision = snap, context, role, revision
        self.records = snap.get("records") if type(snap) is dict else None

    def identity_ok(self) -> bool:
        s = self.s
        return (type(s) is dict and s.get("schema") == CACHE_SCHEMA and s.get("role") == self.role
                and s.get("closed") is True and _int(s.get("process_id"), 1)
                and s.get("qualification") in ("source_bound_candidate", "cpu_source_functions")
                and all(s.get(k) == v for k, v in self.context.items())
                and type(s.get("source")) is dict and s["source"].get("supported") is True
                and s.get("source") == dict(profiles.cache_source(self.revision), supported=True))

    def health_ok(self) -> bool:
        h = self.s.get("health")
        return (type(h) is dict and h.get("complete") is True and h.get("budget_exhausted") is False
                and all(type(h.get(k)) is int and h[k] == 0
                        for k in ("errors", "dropped_records", "late_calls", "active_calls")))

    def budget_ok(self) -> bool:
        lim, recs = self.s.get("budgets"), self.records
        if type(lim) is not dict or not _int(lim.get("max_records"), 1, CACHE_MAX_RECORDS) \
                or not _int(lim.get("max_bytes"), 65536, CACHE_MAX_BYTES):
            return False
        if type(lim.get("retained_records")) is not int or lim["retained_records"] != len(recs):
            return False
        if type(lim.get("retained_bytes")) is not int or lim["retained_bytes"] != sum(len(ev.json_bytes(r)) for r in recs):
            return False
        return (type(lim.get("fixed_bytes")) is int and lim["fixed_bytes"] == CACHE_FIXED_BYTES
                and len(recs) <= lim["max_records"] and lim["retained_bytes"] + CACHE_FIXED_BYTES <= lim["max_bytes"])

    def sequence_ok(self) -> bool:
        seq = [r.get("sequence") if type(r) is dict else None for r in self.records]
        return all(_int(x, 1) for x in seq) and seq == list(range(1, len(seq) + 1))


def _cache_row_findings(row) -> list[str]:
    if (type(row) is not dict or not _text(row.get("request_id")) or not _int(row.get("output_tokens"), 0, MAX_PROMPT_TOKENS)
            or not _int(row.get("preemptions"), 0, MAX_PROMPT_TOKENS) or row.get("status") not in CACHE_STATUSES
            or "stats" not in row):
        return ["native_cache_accounting_record_unverified"]
    v = row["stats"]
    if v is None:
        return []
    counts_ok = (type(v) is dict and set(v) == set(CACHE_FIELDS) and all(_int(v[k], 0, MAX_PROMPT_TOKENS) for k in CACHE_FIELDS)
                 and _int(row.get("prompt_tokens"), 1, MAX_PROMPT_TOKENS)
                 and v["num_prompt_tokens"] == row["prompt_tokens"]
                 and v["num_cached_tokens"] == v["num_local_cached_tokens"] + v["num_external_cached_tokens"]
                 and v["num_prompt_tokens"] == v["num_computed_tokens"] + v["num_cached_tokens"])
    return [] if counts_ok else ["native_cache_accounting_counts_unverified"]


def cache_snapshot(snapshot, context: dict, role: str, revision: str) -> tuple[list, list]:
    """Validated prefill-accounting records of one engine; missing data is never read as zero."""
    c = _CacheSnapshot(snapshot, context, role, revision)
    if not c.identity_ok():
        return [], ["native_cache_accounting_identity_unverified"]
    found = [] if c.health_ok() else ["native_cache_accounting_incomplete"]
    if type(c.records) is not list or len(c.records) > CACHE_MAX_RECORDS:
        return [], found + ["native_cache_accounting_records_unverified"]
    if not c.budget_ok():
        found.append("native_cache_accounting_budget_unverified")
    if not c.sequence_ok():
        found.append("native_cache_accounting_sequence_unverified")
    for row in c.records:
        found += _cache_row_findings(row)
    return c.records, _dedup(found)


def request_usage(records: list, internal_id, prompt_tokens, prompt_sha256, completion_tokens):
    """(first stats, reasons) of one request: exactly one record with stats, monotone output counts ending at the
    client's completion count, a clean finish, and no preemption."""
    mine = [r for r in records if type(r) is dict and r.get("request_id") == internal_id]
    with_stats = [r for r in mine if r.get("stats") is not None]
    if not mine or len(with_stats) != 1:
        return None, ["unambiguous_native_prefill_stats_missing"]
    first = with_stats[0]
    outputs = [r.get("output_tokens") for r in mine]
    found = []
    if first is not mine[0] or first.get("prompt_tokens") != prompt_tokens or first.get("prompt_sha256") != prompt_sha256:
        found.append("native_cache_prompt_binding_unverified")
    terminal_ok = (all(_int(n) for n in outputs) and outputs == sorted(outputs) and _int(completion_tokens, 1)
                   and outputs[-1] == completion_tokens and mine[-1].get("status") in FINISHED_OK
                   and all(r.get("status") == "RUNNING" for r in mine[:-1]))
    if not terminal_ok:
        found.append("native_cache_terminal_request_unverified")
    if any(type(r.get("preemptions")) is not int or r["preemptions"] != 0 for r in mine):
        found.append("native_cache_preempted_request_unsupported")
    return (None if found else first.get("stats")), found
