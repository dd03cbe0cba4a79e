"""Join of a recorded run's three views, per planned client request:

    REQUEST_PLAN.json      (sdcguard.checksum-request-plan.v1)     what the client meant to send, per arm and slot
    CLIENT_INVENTORY.json  (sdcguard.checksum-client-inventory.v1) what each HTTP stage actually sent and got back
    CAPTURES.json          (sdcguard.checksum-client-captures.v1)  what the engines recorded: request-id bindings,
                                                                   checksum observer snapshots, cache accounting

A request passes only if its client stages completed as planned, it binds to exactly one engine-internal request,
that request has exactly one native checksum call, and that call's re-derived scope covers the whole prompt.
Prefix-cache accounting adds the cached-token counts (`join_cache`).

How it is organised. The plan is indexed once (`PlanIndex`, which refuses malformed plans). Every recorded object
is read through a view, and its defects are `Finding`s in ordered tables (observer.Finding): the HTTP stages of a
request (`_STAGE_TABLE`, reasons prefixed by the stage), the transfer descriptor (`_DESCRIPTOR_TABLE`), a binding
snapshot (`_BINDING_TABLE`), an engine capture (`_CAPTURE_TABLE`). The join of one request is a fixed sequence of
steps (`_RequestJoin`), each adding its reasons; a step that cannot proceed ends the sequence.

The reason strings and the join rules are the interface of the recording format and the reference's verdicts
(src/sdcguard/checksum_client.py:274-774, prefix_cache_coverage.py:6-128): the saved recordings must get the same
verdicts.
"""
from __future__ import annotations

import base64
import binascii
import re
from collections import Counter
from typing import Optional

from . import evidence as ev
from . import observer
from . import profiles
from .observer import Finding, _dedup, _int, _run, _text

PLAN_SCHEMA = "sdcguard.checksum-request-plan.v1"
INVENTORY_SCHEMA = "sdcguard.checksum-client-inventory.v1"
CAPTURES_SCHEMA = "sdcguard.checksum-client-captures.v1"
BINDING_SCHEMA = "sdcguard.checksum-request-bindings.v1"
REPORT_SCHEMA = "sdcguard.checksum-client-report.v1"
MAX_REQUESTS, MAX_ARMS, MAX_PHASES, MAX_SNAPSHOTS = 4096, 8, 16, 64
MAX_PROMPT_TOKENS = 8192
CONTEXT_KEYS = ("run_id", "packet_sha256", "arm_id", "engine_session_id")
BINDING_FIXED_BYTES = 8192
PROFILE_LIMITS = ("runtime_qualification_pending", "joint_release_profile_not_qualified")
QUALIFIED = ("source_bound_candidate", "cpu_source_functions")
ROLES = ("prefill", "decode")
HEALTH_ZERO = ("errors", "dropped_records", "late_calls", "active_calls")
_HEX64 = re.compile(r"[0-9a-f]{64}")
_HEX32 = re.compile(r"[0-9a-f]{32}")


def _sha(v) -> bool:
    return type(v) is str and _HEX64.fullmatch(v) is not None


def _is(v, want) -> bool:
    """Typed equality: same Python type as `want` (so True is not 1) and equal."""
    return type(v) is type(want) and v == want


def prompt_digest(tokens) -> str:
    if (type(tokens) is not list or not 1 <= len(tokens) <= MAX_PROMPT_TOKENS
            or not all(_int(t, 0, 2 ** 31 - 1) for t in tokens)):
        raise ev.EvidenceError("prompt must be a bounded nonempty integer token list")
    return ev.digest(ev.json_bytes(tokens))


def _document(raw: bytes, schema: str, what: str) -> dict:
    v = ev.parse_json(raw)
    if type(v) is not dict or v.get("schema") != schema:
        raise ev.EvidenceError("unsupported " + what + " schema")
    return v


def _context(plan: dict, arm: dict) -> dict:
    """The recording context of one arm: the run's identity and the arm's engine session."""
    return {k: plan[k] if k in ("run_id", "packet_sha256") else arm[k] for k in CONTEXT_KEYS}


# ------------------------------------------------------------------------------------------ the plan
class PlanIndex:
    """Every planned request (each slot of each arm) with its arm's session and observer switch, the arms by id
    and the phases' concurrency. A plan that breaks its contract is refused (EvidenceError), never half-read."""

    def __init__(self, plan: dict):
        self.plan = plan
        self._identity()
        self.phases = self._phases(plan.get("phases"))
        self.arms: dict = {}
        self.rows: list = []
        self._arms(plan.get("arms"))

    def _identity(self) -> None:
        p = self.plan
        if "gpu_blocks_override" in p and not _is(p["gpu_blocks_override"], 8192):
            raise ev.EvidenceError("request plan cache capacity is unsupported")
        if type(p.get("prefix_caching", False)) is not bool:
            raise ev.EvidenceError("prefix cache configuration must be a recorded boolean")
        run_id = p.get("run_id")
        if not (type(run_id) is str and _HEX32.fullmatch(run_id) and _sha(p.get("packet_sha256"))
                and profiles.supported(p.get("source_revision")) and _text(p.get("model"))):
            raise ev.EvidenceError("request plan identity, source revision or model is unsupported")

    @staticmethod
    def _phases(phases) -> dict:
        if not isinstance(phases, list) or not 1 <= len(phases) <= MAX_PHASES:
            raise ev.EvidenceError("request plan phases exceed the supported bound")
        out = {}
        for ph in phases:
            ok = type(ph) is dict and _text(ph.get("phase_id"), 128) and _int(ph.get("concurrency"), 1, 64)
            if not ok or ph["phase_id"] in out:
                raise ev.EvidenceError("request plan phase declarations are ambiguous")
            out[ph["phase_id"]] = ph["concurrency"]
        return out

    def _arms(self, arms) -> None:
        if type(arms) is not list or not 1 <= len(arms) <= MAX_ARMS:
            raise ev.EvidenceError("request plan arms exceed the supported bound")
        sessions, ids = set(), set()
        for arm in arms:
            ok = (type(arm) is dict and _text(arm.get("arm_id"), 128) and _text(arm.get("engine_session_id"), 128)
                  and type(arm.get("observer_enabled")) is bool and arm["arm_id"] not in self.arms
                  and arm["engine_session_id"] not in sessions and type(arm.get("requests")) is list
                  and arm["requests"])
            if not ok:
                raise ev.EvidenceError("request plan arm or session declarations are ambiguous")
            self.arms[arm["arm_id"]] = arm
            sessions.add(arm["engine_session_id"])
            for slot, rq in enumerate(arm["requests"]):
                if len(self.rows) >= MAX_REQUESTS:
                    raise ev.EvidenceError("request plan exceeds its logical request bound")
                if not self._request_ok(rq, slot, ids):
                    raise ev.EvidenceError("request plan slot or request contract is malformed")
                ids.update((rq["client_request_id"], rq["prefill_request_id"]))
                self.rows.append({**rq, "arm_id": arm["arm_id"], "engine_session_id": arm["engine_session_id"],
                                  "observer_enabled": arm["observer_enabled"]})
        if not any(a["observer_enabled"] for a in self.arms.values()):
            raise ev.EvidenceError("request plan must retain at least one observed arm")

    def _request_ok(self, rq, slot: int, ids: set) -> bool:
        if type(rq) is not dict or not _is(rq.get("slot"), slot) or not _text(rq.get("phase_id"), 128) \
                or rq["phase_id"] not in self.phases or rq.get("kind") not in ("warmup", "measured"):
            return False
        want_conc = 1 if rq["kind"] == "warmup" else self.phases[rq["phase_id"]]
        cid, pid = rq.get("client_request_id"), rq.get("prefill_request_id")
        return (_int(rq.get("concurrency"), 1, 64) and rq["concurrency"] == want_conc and _text(cid) and _text(pid)
                and cid != pid and cid not in ids and pid not in ids
                and _int(rq.get("prompt_tokens"), 1, MAX_PROMPT_TOKENS) and _sha(rq.get("prompt_sha256"))
                and _int(rq.get("max_tokens"), 1, 4096))


def planned_rows(plan: dict):
    """Flattened planned requests, arms by id, phases by id (PlanIndex); malformed plans raise."""
    ix = PlanIndex(plan)
    return ix.rows, ix.arms, ix.phases


# ------------------------------------------------------------------------------------------ client stages
class _Stage:
    """One HTTP stage (prefill or decode) of a client request as the inventory recorded it."""

    def __init__(self, stage: dict, row: dict, model: str, phase: str):
        self.s, self.row, self.model, self.phase = stage, row, model, phase
        self.body, self.headers, self.resp = stage.get("request_body"), stage.get("request_headers"), \
            stage.get("response_body")
        self.want_id = row["prefill_request_id"] if phase == "prefill" else row["client_request_id"]

    def exchanged(self) -> bool:
        return type(self.body) is dict and type(self.headers) is dict and type(self.resp) is dict

    def completed_200(self) -> bool:
        s = self.s
        return (s.get("completed") is True and "error" in s and s.get("error") is None
                and _is(s.get("http_status"), 200) and s.get("method") == "POST" and s.get("path") == "/v1/completions")

    def id_bound(self) -> bool:
        hdr = [v for k, v in self.headers.items() if type(k) is str and k.lower() == "x-request-id"]
        return hdr == [self.want_id] and self.body.get("request_id") == self.want_id \
            and self.resp.get("id") == "cmpl-" + self.want_id

    def prompt_ok(self) -> bool:
        try:
            dg = prompt_digest(self.body.get("prompt"))
        except ev.EvidenceError:
            dg = None
        usage, n = self.resp.get("usage"), self.row["prompt_tokens"]
        return (dg == self.row["prompt_sha256"] and type(self.body.get("prompt")) is list
                and len(self.body["prompt"]) == n and type(usage) is dict and _is(usage.get("prompt_tokens"), n))

    def single_prompt_api(self) -> bool:
        b = self.body
        want_max = 1 if self.phase == "prefill" else self.row["max_tokens"]
        return (b.get("model") == self.model and _is(b.get("n"), 1) and b.get("stream") is False
                and b.get("add_special_tokens") is False and _is(b.get("max_tokens"), want_max)
                and b.get("use_beam_search", False) is False and b.get("best_of", 1) == 1
                and type(b.get("best_of", 1)) is int)


# (suffix, defect) in order; the reason is "<phase>_<suffix>"
_STAGE_TABLE = (
    Finding("api_request_id_binding_unverified", lambda st: not st.id_bound()),
    Finding("prompt_contract_unverified", lambda st: not st.prompt_ok()),
    Finding("single_prompt_api_contract_unverified", lambda st: not st.single_prompt_api()),
)


def _stage_findings(stage, row, model, phase):
    """(reasons, external request id) of one stage."""
    if type(stage) is not dict:
        return [phase + "_receipt_missing"], None
    st = _Stage(stage, row, model, phase)
    head = [] if st.completed_200() else [phase + "_http_completion_unverified"]
    if not st.exchanged():
        return head + [phase + "_request_or_response_missing"], None
    found = [phase + "_" + r for r in _run(_STAGE_TABLE, st)]
    external = None if not st.id_bound() else st.resp["id"] + "-0"
    return head + found, external


def _b64_nonempty(text) -> bool:
    try:
        return bool(base64.b64decode(text, validate=True))
    except (ValueError, binascii.Error):
        return False


_DESCRIPTOR_TABLE = (   # each entry: the descriptor breaks the transfer contract when it holds
    Finding("direction", lambda d, row: d.get("do_remote_prefill") is not True or d.get("do_remote_decode") is not False),
    Finding("endpoint", lambda d, row: not all(_text(d.get(k)) for k in ("remote_request_id", "remote_engine_id",
                                                                          "remote_host"))
            or not _int(d.get("remote_port"), 1, 65535)),
    Finding("parallel", lambda d, row: not all(_is(d.get(k), 1) for k in ("tp_size", "dcp_size", "pp_size"))),
    Finding("tokens", lambda d, row: not _is(d.get("remote_num_tokens"), row["prompt_tokens"])
            or not _int(d.get("remote_registration_generation"))),
    Finding("blocks", lambda d, row: not (
        type(d.get("remote_block_ids")) is list and len(d["remote_block_ids"]) == 1
        and type(d["remote_block_ids"][0]) is list and 1 <= len(d["remote_block_ids"][0]) <= MAX_PROMPT_TOKENS
        and all(_int(x, 0, 2 ** 64 - 1) for x in d["remote_block_ids"][0]))),
    Finding("checksums", lambda d, row: not _text(d.get("kv_checksums"), 65536) or not _b64_nonempty(d["kv_checksums"])),
)


def _descriptor_ok(d, row) -> bool:
    return type(d) is dict and not any(f.holds(d, row) for f in _DESCRIPTOR_TABLE)


def _client_row(raw, row, model):
    """Reasons and the decode stage's external request id of one inventory row."""
    if type(raw) is not dict:
        return ["client_receipt_missing"], None
    found = []
    if raw.get("arm_id") != row["arm_id"] or not _is(raw.get("slot"), row["slot"]) \
            or raw.get("client_request_id") != row["client_request_id"]:
        found.append("client_plan_slot_binding_unverified")
    p, d = raw.get("prefill"), raw.get("decode")
    found += _stage_findings(p, row, model, "prefill")[0]
    decode_reasons, external = _stage_findings(d, row, model, "decode")
    found += decode_reasons
    if type(p) is not dict or type(d) is not dict:
        return _dedup(found + ["client_transfer_descriptor_binding_unverified"]), external

    def field(obj, key):
        return obj.get(key) if type(obj) is dict else None
    offered = field(p.get("response_body"), "kv_transfer_params")      # what the producer answered
    supplied = field(d.get("request_body"), "kv_transfer_params")     # what the client handed to the consumer
    if not _descriptor_ok(offered, row) or not ev.same(offered, supplied):
        found.append("client_transfer_descriptor_binding_unverified")
    asked = field(p.get("request_body"), "kv_transfer_params")
    if type(asked) is not dict or asked.get("do_remote_decode") is not True or asked.get("do_remote_prefill") is not False:
        found.append("client_prefill_direction_unverified")
    return _dedup(found), external


# ------------------------------------------------------------------------------------------ engine captures
def _ctx_ok(snap, ctx) -> bool:
    return (type(snap) is dict and all(snap.get(k) == ctx[k] for k in CONTEXT_KEYS)
            and _int(snap.get("process_id"), 1, 2 ** 31 - 1))


class _Bindings:
    """One request-id binding snapshot (the engine's external -> internal request ids)."""

    def __init__(self, snap: dict, ctx: dict, revision: str):
        self.s, self.ctx, self.revision = snap, ctx, revision
        q = snap.get("qualification")
        self.qual = q if type(q) is str else None
        recs = snap.get("records")
        self.listed = type(recs) is list
        self.recs = recs if self.listed else []

    def identity_ok(self) -> bool:
        s = self.s
        return (s.get("schema") == BINDING_SCHEMA and s.get("profile") == profiles.BINDING_PROFILE
                and _ctx_ok(s, self.ctx) and s.get("closed") is True and s.get("runtime_qualified") is False
                and s.get("release_qualifying") is False and self.qual in QUALIFIED)

    def source_ok(self) -> bool:
        src = self.s.get("source")
        return (type(src) is dict and src.get("supported") is True and src.get("profile") == profiles.BINDING_PROFILE
                and src.get("revision") == self.revision
                and ev.same(src.get("files"), profiles.get(self.revision)["binding_files"]))

    def health_ok(self) -> bool:
        h = self.s.get("health")
        return (type(h) is dict and h.get("complete") is True and h.get("budget_exhausted") is False
                and all(_is(h.get(k), 0) for k in HEALTH_ZERO))

    def budget_ok(self) -> bool:
        b, n = self.s.get("budgets"), len(self.recs)
        nbytes = sum(len(ev.json_bytes(r)) for r in self.recs)
        return (type(b) is dict and _int(b.get("max_records"), 1, MAX_REQUESTS)
                and _int(b.get("max_bytes"), 65536, 8 * 1024 * 1024) and _is(b.get("retained_records"), n)
                and _is(b.get("retained_bytes"), nbytes) and _is(b.get("fixed_metadata_bytes"), BINDING_FIXED_BYTES)
                and n <= b["max_records"] and nbytes + BINDING_FIXED_BYTES <= b["max_bytes"])

    def sequence_ok(self) -> bool:
        seqs = [r.get("sequence") if type(r) is dict else None for r in self.recs]
        return all(_int(x, 1) for x in seqs) and len(seqs) == len(set(seqs)) and seqs == sorted(seqs)


def _assignment_ok(r) -> bool:
    return (type(r) is dict and _text(r.get("external_request_id"))
            and r.get("external_req_id") == r.get("external_request_id") and _text(r.get("internal_request_id"))
            and r.get("randomization_observed") is True and r.get("native_return_is_none") is True
            and "engine_exception" in r and r.get("engine_exception") is None
            and r.get("external_request_id") != r.get("internal_request_id"))


def _prompt_recorded(r) -> bool:
    return type(r) is dict and _int(r.get("prompt_tokens"), 1, MAX_PROMPT_TOKENS) and _sha(r.get("prompt_sha256"))


_BINDING_TABLE = (
    Finding("binding_snapshot_identity_or_closure_unverified", lambda b: not b.identity_ok()),
    Finding("binding_source_unverified", lambda b: not b.source_ok()),
    Finding("binding_recording_health_unverified", lambda b: not b.health_ok()),
    Finding("binding_record_list_unverified", lambda b: not b.listed),
)


def bindings(snapshot, ctx, revision=profiles.BASELINE):
    """(records, reasons, qualification) of one request-id binding snapshot."""
    if type(snapshot) is not dict:
        return [], ["binding_snapshot_missing"], None
    b = _Bindings(snapshot, ctx, revision)
    found = _run(_BINDING_TABLE, b)
    if len(b.recs) > MAX_REQUESTS:
        raise ev.EvidenceError("binding records exceed the supported bound")
    if not b.budget_ok():
        found.append("binding_snapshot_budget_unverified")
    if not b.sequence_ok():
        found.append("binding_sequence_unverified")
    for r in b.recs:
        if not _assignment_ok(r):
            found.append("binding_native_assignment_unverified")
        if not _prompt_recorded(r):
            found.append("native_prompt_recording_unverified")
    return b.recs, _dedup(found), b.qual


class _Capture:
    """One engine capture of an observed arm: startup, binding snapshots, checksum snapshots."""

    def __init__(self, value: dict, plan: dict, arm: dict):
        self.v, self.plan = value, plan
        self.revision = profiles.get(plan["source_revision"])["revision"]
        self.ctx = _context(plan, arm)

    def identity_ok(self) -> bool:
        v = self.v
        return (all(v.get(k) == self.ctx[k] for k in ("arm_id", "engine_session_id"))
                and v.get("source_revision") == self.revision and v.get("capture_complete") is True)

    def startup_ok(self) -> bool:
        v, st = self.v, self.v.get("startup")
        return (type(st) is dict and _sha(v.get("startup_sha256")) and ev.digest(ev.json_bytes(st)) == v["startup_sha256"]
                and all(st.get(k) == self.ctx[k] for k in CONTEXT_KEYS) and st.get("source_revision") == self.revision
                and st.get("role") == "decode" and st.get("model") == self.plan["model"]
                and ev.same(st.get("source_profile"), profiles.client_source(self.revision))
                and st.get("checksum_enabled") is True and st.get("request_id_randomization_enabled") is True)


_CAPTURE_TABLE = (
    Finding("engine_capture_identity_or_closure_unverified", lambda c: not c.identity_ok()),
    Finding("engine_startup_binding_unverified", lambda c: not c.startup_ok()),
    Finding("binding_snapshot_list_unverified", lambda c: type(c.v.get("binding_snapshots")) is not list),
    Finding("checksum_snapshot_list_unverified", lambda c: type(c.v.get("checksum_snapshots")) is not list),
)
# hold reasons of one snapshot's report that say nothing about the capture (the join establishes or reports them)
_REPORT_ONLY = set(observer.REPORT_LIMITS) | {"no_recorded_native_verification_calls"}


def _empty_facts(issues: list, qualification: str) -> dict:
    return {"issues": issues, "bindings": [], "calls": [], "unverified": [], "qualification": qualification}


def _capture(value, plan, arm) -> dict:
    """Facts of one engine capture: its issues, binding records, re-derived checksum calls, unverified
    observations and the qualification domain every snapshot agrees on."""
    if type(value) is not dict:
        return _empty_facts(["engine_capture_missing"], "unknown")
    c = _Capture(value, plan, arm)
    found = _run(_CAPTURE_TABLE, c)
    bsnaps = value["binding_snapshots"] if type(value.get("binding_snapshots")) is list else []
    csnaps = value["checksum_snapshots"] if type(value.get("checksum_snapshots")) is list else []
    if len(bsnaps) > MAX_SNAPSHOTS or len(csnaps) > MAX_SNAPSHOTS:
        raise ev.EvidenceError("capture snapshot lists exceed the supported bound")
    facts = _empty_facts([], "unknown")
    domains, active_b, active_c, nrec = [], 0, 0, 0
    for i, snap in enumerate(bsnaps):
        recs, issues, dom = bindings(snap, c.ctx, c.revision)
        found += issues
        domains.append(dom)
        active_b += bool(recs)
        facts["bindings"] += [{**r, "binding_snapshot_index": i, "process_id": snap.get("process_id")}
                              for r in recs if type(r) is dict]
        if len(facts["bindings"]) > MAX_REQUESTS:
            raise ev.EvidenceError("aggregate binding records exceed the supported bound")
    for i, snap in enumerate(csnaps):
        if type(snap) is dict and type(snap.get("records")) is list:
            nrec += len(snap["records"])
            if nrec > MAX_REQUESTS:
                raise ev.EvidenceError("aggregate checksum records exceed the supported bound")
        if type(snap) is not dict or not _ctx_ok(snap.get("capture_context"), c.ctx):
            found.append("checksum_capture_context_unverified")
        try:
            rep = observer.snapshot_report(ev.parse_json(ev.json_bytes(snap)), revision=c.revision)
        except (ev.EvidenceError, TypeError, ValueError) as e:
            found.append("checksum_snapshot_unreadable")
            facts["unverified"].append({"request_id": None, "reason": "checksum_snapshot_unreadable",
                                        "detail": type(e).__name__})
            continue
        dom = rep["qualification"]
        domains.append(dom if type(dom) is str else None)
        found += [x for x in rep["hold_reasons"] if x not in _REPORT_ONLY]
        active_c += bool(snap.get("records"))
        cctx = snap.get("capture_context")
        for call in rep["verification_calls"]:
            orig = snap["records"][call["record_index"]]
            proof = orig.get("proof") if type(orig) is dict else None
            facts["calls"].append({**call, "checksum_snapshot_index": i,
                                   "checksum_num_tokens": proof.get("num_tokens") if type(proof) is dict else None,
                                   "process_id": cctx.get("process_id") if type(cctx) is dict else None})
        facts["unverified"] += rep["unverified_observations"]
    if active_b != 1:
        found.append("unambiguous_active_binding_recorder_missing")
    if active_c != 1:
        found.append("unambiguous_active_checksum_recorder_missing")
    one_domain = bool(domains) and len(set(domains)) == 1
    if not one_domain or domains[0] not in QUALIFIED:
        found.append("capture_qualification_domain_unverified")
    facts["issues"] = _dedup(found)
    facts["qualification"] = domains[0] if one_domain else "unknown"
    return facts


# ------------------------------------------------------------------------------------------ cache accounting join
def _role_envelope(capture: dict, role: str) -> dict:
    env = capture.get("prefill_capture") if role == "prefill" else capture
    return env if type(env) is dict else {}


def _cache_startup_ok(st: dict, role: str, ctx: dict, plan: dict) -> bool:
    rev = plan["source_revision"]
    return (st.get("role") == role and all(st.get(k) == v for k, v in ctx.items()) and st.get("prefix_caching") is True
            and st.get("checksum_enabled") is True and st.get("source_revision") == rev
            and profiles.startup_supported(st, rev))


def cache_facts(capture, plan, arm) -> dict:
    """Per role (prefill, decode): the engine's prefill-accounting records, its binding records, the issues of
    both, and the internal ids joined so far (filled by `cache_usage`)."""
    ctx = _context(plan, arm)
    out = {}
    for role in ROLES:
        env = _role_envelope(capture, role)
        st = env.get("startup", {})
        st = st if type(st) is dict else {}
        found, recs, binds = [], [], []
        if not _cache_startup_ok(st, role, ctx, plan):
            found.append("native_cache_startup_unverified:" + role)
        snaps = env.get("cache_snapshots")
        single = snaps[0] if type(snaps) is list and len(snaps) == 1 else None
        if type(snaps) is not list or len(snaps) != 1:
            found.append("native_cache_snapshot_missing_or_ambiguous:" + role)
        else:
            recs, errs = observer.cache_snapshot(single, ctx, role, plan["source_revision"])
            found += errs
            if type(single) is not dict or single.get("process_id") != st.get("process_id"):
                found.append("native_cache_process_binding_unverified:" + role)
        bsnaps = env.get("binding_snapshots")
        if type(bsnaps) is not list or len(bsnaps) > MAX_SNAPSHOTS:
            found.append("cache_request_binding_snapshots_missing:" + role)
        else:
            active = 0
            for snap in bsnaps:
                rows, errs, dom = bindings(snap, ctx, plan["source_revision"])
                found += errs
                active += bool(rows)
                binds += rows
                if type(single) is dict and dom != single.get("qualification"):
                    found.append("native_cache_qualification_disagrees:" + role)
                if len(binds) > MAX_REQUESTS:
                    raise ev.EvidenceError("native cache bindings exceed their bound")
            if active != 1:
                found.append("cache_request_binding_ambiguous:" + role)
        out[role] = {"records": recs, "bindings": binds, "issues": _dedup(found), "joined": set()}
    return out


def _cache_binding(f: dict, row: dict, role: str, strict: bool) -> Optional[str]:
    """The engine-internal id the role's binding records give this request, or None when the join fails."""
    rid = row["prefill_request_id"] if role == "prefill" else row["client_request_id"]
    hits = [b for b in f["bindings"] if b.get("external_request_id") == "cmpl-" + rid + "-0"]
    if len(hits) != 1:
        return None
    b = hits[0]
    internal = b.get("internal_request_id")
    if strict and (type(internal) is not str or not internal):
        return None
    if sum(x.get("internal_request_id") == internal for x in f["bindings"]) != 1:
        return None
    if b.get("prompt_sha256") != row["prompt_sha256"]:
        return None
    if (strict and type(b.get("prompt_tokens")) is not int) or b.get("prompt_tokens") != row["prompt_tokens"]:
        return None
    if role == "decode" and internal != row.get("internal_request_id"):
        return None
    return internal


def _response_of(raw, role: str) -> dict:
    stage = raw.get(role, {}) if type(raw) is dict else {}
    resp = stage.get("response_body", {}) if type(stage) is dict else {}
    return resp if type(resp) is dict else {}


def _producer_counts_ok(desc, internal, stats: dict) -> bool:
    """The producer's transfer descriptor names the joined request and reports the cached tokens it accounted."""
    return (type(desc) is dict and desc.get("remote_request_id") == internal and stats["num_external_cached_tokens"] == 0
            and _is(desc.get("remote_prefill_cached_tokens"), stats["num_cached_tokens"]))


def cache_usage(facts: dict, raw, row: dict, *, for_transfer: bool = False):
    """Per-role cache stats of one request joined through the binding records. Returns (stats by role, issues).
    for_transfer: the stricter join of the transfer-only view (an unusable role contributes no stats)."""
    stats, issues = {}, []
    for role in ROLES:
        f = facts[role]
        issues += f["issues"]
        internal = _cache_binding(f, row, role, strict=for_transfer)
        if internal is None:
            issues.append("native_cache_request_join_unverified:" + role)
            continue
        f["joined"].add(internal)
        resp = _response_of(raw, role)
        usage = resp.get("usage", {})
        usage = usage if type(usage) is dict else {}
        value, errs = observer.request_usage(f["records"], internal, row["prompt_tokens"], row["prompt_sha256"],
                                             usage.get("completion_tokens"))
        issues += [e + ":" + role for e in errs]
        usable = not f["issues"] and not errs and type(value) is dict
        desc = resp.get("kv_transfer_params", {})
        if for_transfer:
            if not usable:
                continue
            if role == "prefill" and not _producer_counts_ok(desc, internal, value):
                issues.append("producer_cache_descriptor_counts_unverified")
                continue
            stats[role] = value
            continue
        if role == "prefill":
            if type(desc) is not dict or desc.get("remote_request_id") != internal:
                issues.append("producer_cache_transfer_request_binding_unverified")
            if usable:
                cached = desc.get("remote_prefill_cached_tokens") if type(desc) is dict else None
                if value["num_external_cached_tokens"] != 0 or not _is(cached, value["num_cached_tokens"]):
                    issues.append("producer_cache_descriptor_counts_unverified")
                    usable = False
        if usable:
            stats[role] = value
    return stats, _dedup(issues)


def join_cache(facts, raw, row):
    """Token coverage of one request from cache accounting and its checksum call (full-prompt view)."""
    usage = {"prompt_tokens": row["prompt_tokens"], "transferred_tokens_checked": None,
             "decode_cached_tokens_unchecked": None, "decode_locally_computed_tokens": None,
             "prefill_cached_tokens": None, "prefill_reused_cached_blocks": "unknown"}
    stats, errors = cache_usage(facts, raw, row)
    if "prefill" in stats:
        n = stats["prefill"]["num_local_cached_tokens"]
        usage.update(prefill_cached_tokens=n, prefill_reused_cached_blocks=n > 0)
    if "decode" not in stats:
        return usage, _dedup(errors)
    v = stats["decode"]
    local, remote, computed = v["num_local_cached_tokens"], v["num_external_cached_tokens"], v["num_computed_tokens"]
    usage.update(decode_cached_tokens_unchecked=local, decode_locally_computed_tokens=computed)
    if local:
        errors.append(observer.CACHED_PREFIX_REASON)
    if computed:
        errors.append("locally_computed_prompt_not_covered_by_checksum")
    calls = row.get("checksum_calls", [])
    scope = calls[0].get("conditional_scope", {}).get("token_coverage", {}) if len(calls) == 1 else {}
    span_agrees = (len(calls) == 1 and not calls[0].get("recording_issues")
                   and scope.get("prompt_tokens") == row["prompt_tokens"]
                   and scope.get("decode_cached_tokens_unchecked") == local
                   and scope.get("transferred_tokens_checked") == remote and remote == row["prompt_tokens"] - local)
    if span_agrees:
        usage["transferred_tokens_checked"] = remote
    elif not calls and remote == 0:
        usage["transferred_tokens_checked"] = 0
        errors.append("no_transfer_checksum_comparison_recorded")
    else:
        errors.append("native_cache_to_checksum_span_unverified")
    return usage, _dedup(errors)


def unexpected_cache(facts) -> list[str]:
    """Roles whose accounting or bindings name internal requests no planned request joined."""
    out = []
    for role, f in facts.items():
        seen = {r.get("request_id") for r in f["records"] if type(r) is dict and type(r.get("request_id")) is str}
        bound = {r.get("internal_request_id") for r in f["bindings"] if type(r.get("internal_request_id")) is str}
        if (seen | bound) - f["joined"]:
            out.append("unexpected_native_cache_requests:" + role)
    return out


# ------------------------------------------------------------------------------------------ the join
def _row_template(rq: dict, reasons: list, external) -> dict:
    row = dict(rq)
    row.update(client_status="complete" if not reasons else "unknown", external_request_id=external,
               internal_request_id=None, binding_status="unknown", native_result="unverified", coverage="unknown",
               check_status="unverified", checksum_calls=[], unverified_observations=[], reasons=reasons)
    row["token_coverage"] = {"prompt_tokens": row["prompt_tokens"], "transferred_tokens_checked": None,
                             "decode_cached_tokens_unchecked": None, "decode_locally_computed_tokens": None,
                             "prefill_cached_tokens": None, "prefill_reused_cached_blocks": "unknown"}
    return row


class _RequestJoin:
    """Joins one planned request to its engine facts: binding, then the checksum call. Each step appends its
    reasons to the row; `joined_bindings` / `joined_calls` collect what a matched request accounted for."""

    def __init__(self, row: dict, facts: dict, joined_bindings: set, joined_calls: set):
        self.row, self.f = row, facts
        self.joined_bindings, self.joined_calls = joined_bindings, joined_calls

    def run(self) -> None:
        b = self._binding()
        if b is None:
            return
        self._calls(b)

    def _binding(self) -> Optional[dict]:
        row, f = self.row, self.f
        ext = row["external_request_id"]
        hits = [b for b in f["bindings"] if b.get("external_request_id") == ext] if ext else []
        if len(hits) != 1:
            row["reasons"].append("unambiguous_native_request_binding_missing")
            return None
        b = hits[0]
        internal = b.get("internal_request_id")
        if not _text(internal) or not _int(b.get("sequence"), 1):
            row["reasons"].append("native_request_binding_identity_unverified")
            return None
        if sum(x.get("internal_request_id") == internal for x in f["bindings"]) != 1:
            row["reasons"].append("native_internal_request_binding_ambiguous")
            return None
        row["internal_request_id"] = internal
        if b.get("prompt_sha256") != row["prompt_sha256"] or not _is(b.get("prompt_tokens"), row["prompt_tokens"]):
            row["reasons"].append("native_prompt_to_client_binding_unverified")
        if row["client_status"] == "complete" and not row["reasons"]:
            row["binding_status"] = "matched"
            self.joined_bindings.add((row["arm_id"], b.get("capture_index"), b["binding_snapshot_index"], b["sequence"]))
        return b

    def _calls(self, b: dict) -> None:
        row, f = self.row, self.f
        internal = row["internal_request_id"]
        row["unverified_observations"] = [e for e in f["unverified"] if e.get("request_id") == internal]
        row["reasons"] += [e["reason"] for e in row["unverified_observations"] if _text(e.get("reason"))]
        mine = [(i, c) for i, c in enumerate(f["calls"]) if c.get("request_id") == internal]
        row["checksum_calls"] = [c for _, c in mine]
        if row["binding_status"] == "matched":
            self.joined_calls.update((row["arm_id"], i) for i, _ in mine)
        if len(mine) != 1:
            row["reasons"].append("unambiguous_native_checksum_call_missing")
            return
        c = mine[0][1]
        row["native_result"] = c["native_result"]
        if c["coverage"] != "complete":
            row["reasons"].append(c["engine_pass_not_covered_reason"] or c["reason"])
        if not _is(c.get("checksum_num_tokens"), row["prompt_tokens"]):
            row["reasons"].append("client_prompt_to_checksum_span_unverified")
        if not row["reasons"] and row["binding_status"] == "matched" and c["coverage"] == "complete":
            row["coverage"] = "complete"
            row["check_status"] = "passed" if c["native_result"] == "passed" else "mismatch"
            if row["check_status"] == "mismatch":
                row["reasons"].append("native_checksum_mismatch")


def _tag(facts: dict, idx: int) -> dict:
    for k in ("bindings", "calls", "unverified"):
        facts[k] = [{**e, "capture_index": idx} for e in facts[k]]
    return facts


def _merge(parsed: list) -> dict:
    """Facts of an arm with several captures: everything of each, held as ambiguous."""
    merged = _empty_facts(_dedup(["ambiguous_engine_captures"] + [x for p in parsed for x in p["issues"]]), "unknown")
    for k in ("bindings", "calls", "unverified"):
        merged[k] = [e for p in parsed for e in p[k]]
    return merged


def _orphan_arm(raw, i: int) -> dict:
    aid = raw.get("arm_id") if type(raw) is dict else None
    sid = raw.get("engine_session_id") if type(raw) is dict else None
    return {"arm_id": aid if _text(aid, 128) else "unknown-capture-" + str(i),
            "engine_session_id": sid if _text(sid, 128) else "unknown-session"}


def evaluate(plan_raw: bytes, inventory_raw: bytes, captures_raw: bytes) -> dict:
    plan = _document(plan_raw, PLAN_SCHEMA, "checksum request plan")
    inventory = _document(inventory_raw, INVENTORY_SCHEMA, "checksum client inventory")
    captures = _document(captures_raw, CAPTURES_SCHEMA, "checksum client captures")
    ix = PlanIndex(plan)
    plan_sha = ev.digest(plan_raw)

    def bound(v) -> bool:
        return (v.get("run_id") == plan.get("run_id") and v.get("packet_sha256") == plan.get("packet_sha256")
                and v.get("plan_sha256") == plan_sha)
    inv_ok, cap_ok = bound(inventory), bound(captures)
    issues = [reason for reason, bad in (("client_inventory_run_binding_unverified", not inv_ok),
                                         ("client_inventory_completion_unverified", inventory.get("completed") is not True),
                                         ("capture_manifest_run_binding_unverified", not cap_ok)) if bad]
    inv_rows = inventory.get("requests")
    if type(inv_rows) is not list:
        issues.append("client_inventory_row_list_unverified")
        inv_rows = []
    if len(inv_rows) > MAX_REQUESTS:
        raise ev.EvidenceError("client inventory rows exceed the supported bound")
    cap_list = captures.get("captures")
    if type(cap_list) is not list:
        issues.append("capture_list_unverified")
        cap_list = []
    if len(cap_list) > MAX_ARMS:
        raise ev.EvidenceError("client capture arms exceed the supported bound")

    # inventory rows by planned (arm, slot)
    planned_keys = {(r["arm_id"], r["slot"]) for r in ix.rows}
    by_slot, stray_rows = {}, []
    for i, raw in enumerate(inv_rows):
        key = (raw.get("arm_id"), raw.get("slot")) if type(raw) is dict else None
        if key is not None and type(key[0]) is str and type(key[1]) is int and key in planned_keys:
            by_slot.setdefault(key, []).append(raw)
        else:
            stray_rows.append(i)
    if stray_rows:
        issues.append("unexpected_client_inventory_rows")

    # captures by observed arm; the rest become facts of their own, held as outside the plan
    by_arm, strays = {}, []
    for i, raw in enumerate(cap_list):
        aid = raw.get("arm_id") if type(raw) is dict else None
        if type(aid) is str and aid in ix.arms and ix.arms[aid]["observer_enabled"] is True:
            by_arm.setdefault(aid, []).append((i, raw))
            continue
        orphan = _orphan_arm(raw, i)
        f = _tag(_capture(raw, plan, orphan), i)
        f["issues"].append("capture_outside_observed_arm")
        strays.append((orphan["arm_id"], f))
    if strays:
        issues.append("unexpected_engine_captures")

    arm_facts, cache = {}, {}
    for name, arm in ix.arms.items():
        if arm["observer_enabled"] is False:
            arm_facts[name] = _empty_facts([], "observer_disabled")
            continue
        mine = by_arm.get(name, [])
        parsed = [_tag(_capture(raw, plan, arm), i) for i, raw in mine]
        f = parsed[0] if len(parsed) == 1 else _capture(None, plan, arm) if not parsed else _merge(parsed)
        if not cap_ok:
            f["issues"].append("capture_manifest_run_binding_unverified")
        arm_facts[name] = f
        if plan.get("prefix_caching") is True:
            cache[name] = cache_facts(mine[0][1] if len(mine) == 1 else {}, plan, arm)
    every = [(n, f, False) for n, f in arm_facts.items()] + [(n, f, True) for n, f in strays]

    rows, joined_calls, joined_binds = [], set(), set()
    for rq in ix.rows:
        mine = by_slot.get((rq["arm_id"], rq["slot"]), [])
        raw = mine[0] if len(mine) == 1 else None
        reasons, external = _client_row(raw, rq, plan["model"])
        if len(mine) > 1:
            reasons.append("ambiguous_client_receipts")
        if not inv_ok:
            reasons.append("client_inventory_run_binding_unverified")
        row = _row_template(rq, reasons, external)
        if row["observer_enabled"] is False:
            row["binding_status"] = "observer_disabled"
            row["reasons"].append("observer_disabled")
            rows.append(row)
            continue
        f = arm_facts[row["arm_id"]]
        row["reasons"] += f["issues"]
        _RequestJoin(row, f, joined_binds, joined_calls).run()
        calls = row["checksum_calls"]
        if plan.get("prefix_caching") is True:
            row["token_coverage"], extra = join_cache(cache[row["arm_id"]], raw, row)
            row["reasons"] += extra
            if extra:
                tc = row["token_coverage"]
                partly = (tc["decode_cached_tokens_unchecked"] and type(tc["transferred_tokens_checked"]) is int
                          and tc["transferred_tokens_checked"] > 0)
                row["coverage"] = "partial" if partly else "unknown"
                row["check_status"] = "unverified"
        elif len(calls) == 1 and not calls[0].get("recording_issues"):
            row["token_coverage"].update(calls[0]["conditional_scope"]["token_coverage"])
        if row["native_result"] == "mismatch":
            row["reasons"].append("native_checksum_mismatch")
        row["reasons"] = _dedup(row["reasons"])
        if not calls:
            row["reasons"].append("no_recorded_checksum_call_for_client_request")
        rows.append(row)

    stray_calls = stray_binds = False
    for aid, f, outside in every:
        for b in f["bindings"]:
            s = b.get("sequence")
            key = (aid, b.get("capture_index"), b["binding_snapshot_index"], s) if _int(s, 1) else None
            stray_binds = stray_binds or outside or key is None or key not in joined_binds
        stray_calls = stray_calls or any(outside or (aid, i) not in joined_calls for i in range(len(f["calls"])))
    if stray_calls:
        issues.append("unexpected_checksum_calls")
    if stray_binds:
        issues.append("unexpected_native_request_bindings")
    for f in cache.values():
        issues += unexpected_cache(f)
    complete = sum(r["client_status"] == "complete" for r in rows)
    if not (inv_ok and inventory.get("completed") is True and not stray_rows and complete == len(rows)):
        issues.append("client_inventory_incomplete")
    open_requests = sum(r["observer_enabled"] and r["check_status"] != "passed" for r in rows)
    if open_requests:
        issues.append("required_checksum_coverage_incomplete")
    summary = {"declared_requests": len(rows), "joined_requests": sum(r["binding_status"] == "matched" for r in rows),
               "checksum_calls": sum(len(f["calls"]) for _, f, _ in every), "joined_checksum_calls": len(joined_calls),
               "native_results": dict(Counter(c["native_result"] for _, f, _ in every for c in f["calls"])),
               "verified_on_requests": sum(r["check_status"] == "passed" for r in rows),
               "on_unverified_requests": open_requests}
    return {"schema": REPORT_SCHEMA, "source_revision": plan["source_revision"], "summary": summary, "requests": rows,
            "captures": [{"arm_id": n, "qualification": f["qualification"], "issues": f["issues"],
                          "planned_arm": not outside} for n, f, outside in every],
            "hold_reasons": _dedup(issues + list(PROFILE_LIMITS))}
