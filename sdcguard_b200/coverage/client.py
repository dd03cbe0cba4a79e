"""Join of a recorded run's three views, per planned client request:

    REQUEST_PLAN.json      (sdcguard.checksum-request-plan.v1)     what the client meant to send, per arm and slot
    CLIENT_INVENTORY.json  (sdcguard.checksum-client-inventory.v1) what each HTTP stage actually sent and got back
    CAPTURES.json          (sdcguard.checksum-client-captures.v1)  what the engines recorded: request-id bindings,
                                                                   checksum observer snapshots, cache accounting

A request passes only if its client stages completed as planned, it binds to exactly one engine-internal request,
that request has exactly one native checksum call, and that call's re-derived scope covers the whole prompt.
Prefix-cache accounting adds the cached-token counts (`join_cache`).

The reason strings and the join rules are the interface of the recording format and the reference's verdicts
(src/sdcguard/checksum_client.py:274-774, prefix_cache_coverage.py:6-128); this is this package's own code.
"""
from __future__ import annotations

import base64
import binascii
import re
from collections import Counter

from . import evidence as ev
from . import observer
from . import profiles

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


def _text(v, n=1024):
    return type(v) is str and 0 < len(v) <= n and "\x00" not in v


def _int(v, lo=0, hi=2 ** 63 - 1):
    return type(v) is int and lo <= v <= hi


def _sha(v):
    return type(v) is str and re.fullmatch(r"[0-9a-f]{64}", v) is not None


def prompt_digest(tokens) -> str:
    if (type(tokens) is not list or not 1 <= len(tokens) <= MAX_PROMPT_TOKENS
            or any(not _int(t, 0, 2 ** 31 - 1) for t in tokens)):
        raise ev.EvidenceError("prompt must be a bounded nonempty integer token list")
    return ev.digest(ev.json_bytes(tokens))


def _read(raw, schema, what):
    v = ev.parse_json(raw)
    if type(v) is not dict or v.get("schema") != schema:
        raise ev.EvidenceError("unsupported " + what + " schema")
    return v


def _bound_to(plan, v, plan_raw) -> bool:
    return (v.get("run_id") == plan.get("run_id") and v.get("packet_sha256") == plan.get("packet_sha256")
            and v.get("plan_sha256") == ev.digest(plan_raw))


def planned_rows(plan: dict):
    """Flattened planned requests (every slot of every arm), arms by id, phases by id; malformed plans raise."""
    if "gpu_blocks_override" in plan and (type(plan["gpu_blocks_override"]) is not int
                                          or plan["gpu_blocks_override"] != 8192):
        raise ev.EvidenceError("request plan cache capacity is unsupported")
    if type(plan.get("prefix_caching", False)) is not bool:
        raise ev.EvidenceError("prefix cache configuration must be a recorded boolean")
    if (type(plan.get("run_id")) is not str or re.fullmatch(r"[0-9a-f]{32}", plan["run_id"]) is None
            or not _sha(plan.get("packet_sha256")) or not profiles.supported(plan.get("source_revision"))
            or not _text(plan.get("model"))):
        raise ev.EvidenceError("request plan identity, source revision or model is unsupported")
    phases, arms = plan.get("phases"), plan.get("arms")
    if not isinstance(phases, list) or not 1 <= len(phases) <= MAX_PHASES:
        raise ev.EvidenceError("request plan phases exceed the supported bound")
    pmap = {}
    for ph in phases:
        if (type(ph) is not dict or not _text(ph.get("phase_id"), 128) or not _int(ph.get("concurrency"), 1, 64)
                or ph["phase_id"] in pmap):
            raise ev.EvidenceError("request plan phase declarations are ambiguous")
        pmap[ph["phase_id"]] = ph["concurrency"]
    if type(arms) is not list or not 1 <= len(arms) <= MAX_ARMS:
        raise ev.EvidenceError("request plan arms exceed the supported bound")
    rows, amap, ids, sessions = [], {}, set(), set()
    for arm in arms:
        if (type(arm) is not dict or not _text(arm.get("arm_id"), 128) or not _text(arm.get("engine_session_id"), 128)
                or type(arm.get("observer_enabled")) is not bool or arm["arm_id"] in amap
                or arm["engine_session_id"] in sessions or type(arm.get("requests")) is not list or not arm["requests"]):
            raise ev.EvidenceError("request plan arm or session declarations are ambiguous")
        amap[arm["arm_id"]] = arm
        sessions.add(arm["engine_session_id"])
        for slot, rq in enumerate(arm["requests"]):
            if len(rows) >= MAX_REQUESTS:
                raise ev.EvidenceError("request plan exceeds its logical request bound")
            if (type(rq) is not dict or type(rq.get("slot")) is not int or rq["slot"] != slot
                    or not _text(rq.get("phase_id"), 128) or rq["phase_id"] not in pmap
                    or rq.get("kind") not in ("warmup", "measured") or not _int(rq.get("concurrency"), 1, 64)
                    or rq["concurrency"] != (1 if rq["kind"] == "warmup" else pmap[rq["phase_id"]])
                    or not _text(rq.get("client_request_id")) or not _text(rq.get("prefill_request_id"))
                    or rq["client_request_id"] == rq["prefill_request_id"] or rq["client_request_id"] in ids
                    or rq["prefill_request_id"] in ids or not _int(rq.get("prompt_tokens"), 1, MAX_PROMPT_TOKENS)
                    or not _sha(rq.get("prompt_sha256")) or not _int(rq.get("max_tokens"), 1, 4096)):
                raise ev.EvidenceError("request plan slot or request contract is malformed")
            ids.update((rq["client_request_id"], rq["prefill_request_id"]))
            rows.append({**rq, "arm_id": arm["arm_id"], "engine_session_id": arm["engine_session_id"],
                         "observer_enabled": arm["observer_enabled"]})
    if not any(a["observer_enabled"] for a in amap.values()):
        raise ev.EvidenceError("request plan must retain at least one observed arm")
    return rows, amap, pmap


# ------------------------------------------------------------------------------------------ client stages
def _stage(stage, row, model, phase):
    if type(stage) is not dict:
        return [phase + "_receipt_missing"], None
    R, external = [], None
    if (stage.get("completed") is not True or "error" not in stage or stage.get("error") is not None
            or type(stage.get("http_status")) is not int or stage["http_status"] != 200
            or stage.get("method") != "POST" or stage.get("path") != "/v1/completions"):
        R.append(phase + "_http_completion_unverified")
    body, headers, resp = stage.get("request_body"), stage.get("request_headers"), stage.get("response_body")
    if type(body) is not dict or type(headers) is not dict or type(resp) is not dict:
        return R + [phase + "_request_or_response_missing"], None
    want = row["prefill_request_id"] if phase == "prefill" else row["client_request_id"]
    hdr = [v for k, v in headers.items() if type(k) is str and k.lower() == "x-request-id"]
    if hdr != [want] or body.get("request_id") != want or resp.get("id") != "cmpl-" + want:
        R.append(phase + "_api_request_id_binding_unverified")
    else:
        external = resp["id"] + "-0"
    try:
        dg = prompt_digest(body.get("prompt"))
    except ev.EvidenceError:
        dg = None
    usage = resp.get("usage")
    if (dg != row["prompt_sha256"] or type(body.get("prompt")) is not list or len(body["prompt"]) != row["prompt_tokens"]
            or type(usage) is not dict or type(usage.get("prompt_tokens")) is not int
            or usage["prompt_tokens"] != row["prompt_tokens"]):
        R.append(phase + "_prompt_contract_unverified")
    mt = 1 if phase == "prefill" else row["max_tokens"]
    if (body.get("model") != model or type(body.get("n")) is not int or body["n"] != 1 or body.get("stream") is not False
            or body.get("add_special_tokens") is not False or type(body.get("max_tokens")) is not int
            or body["max_tokens"] != mt or body.get("use_beam_search", False) is not False
            or body.get("best_of", 1) != 1 or type(body.get("best_of", 1)) is not int):
        R.append(phase + "_single_prompt_api_contract_unverified")
    return R, external


def _descriptor_ok(v, row) -> bool:
    if type(v) is not dict:
        return False
    blocks = v.get("remote_block_ids")
    if (v.get("do_remote_prefill") is not True or v.get("do_remote_decode") is not False
            or any(not _text(v.get(k)) for k in ("remote_request_id", "remote_engine_id", "remote_host"))
            or not _int(v.get("remote_port"), 1, 65535)
            or any(type(v.get(k)) is not int or v[k] != 1 for k in ("tp_size", "dcp_size", "pp_size"))
            or type(v.get("remote_num_tokens")) is not int or v["remote_num_tokens"] != row["prompt_tokens"]
            or not _int(v.get("remote_registration_generation")) or type(blocks) is not list or len(blocks) != 1
            or type(blocks[0]) is not list or not 1 <= len(blocks[0]) <= MAX_PROMPT_TOKENS
            or any(not _int(x, 0, 2 ** 64 - 1) for x in blocks[0]) or not _text(v.get("kv_checksums"), 65536)):
        return False
    try:
        return bool(base64.b64decode(v["kv_checksums"], validate=True))
    except (ValueError, binascii.Error):
        return False


def _client_row(raw, row, model):
    if type(raw) is not dict:
        return ["client_receipt_missing"], None
    R = []
    if (raw.get("arm_id") != row["arm_id"] or type(raw.get("slot")) is not int or raw["slot"] != row["slot"]
            or raw.get("client_request_id") != row["client_request_id"]):
        R.append("client_plan_slot_binding_unverified")
    pr, _ = _stage(raw.get("prefill"), row, model, "prefill")
    dr, external = _stage(raw.get("decode"), row, model, "decode")
    R.extend(pr + dr)
    p, d = raw.get("prefill"), raw.get("decode")
    if type(p) is dict and type(d) is dict:
        resp, body = p.get("response_body"), d.get("request_body")
        desc = resp.get("kv_transfer_params") if type(resp) is dict else None
        supplied = body.get("kv_transfer_params") if type(body) is dict else None
        if not _descriptor_ok(desc, row) or not ev.same(desc, supplied):
            R.append("client_transfer_descriptor_binding_unverified")
        pb = p.get("request_body")
        opts = pb.get("kv_transfer_params") if type(pb) is dict else None
        if type(opts) is not dict or opts.get("do_remote_decode") is not True or opts.get("do_remote_prefill") is not False:
            R.append("client_prefill_direction_unverified")
    else:
        R.append("client_transfer_descriptor_binding_unverified")
    return list(dict.fromkeys(R)), external


# ------------------------------------------------------------------------------------------ engine captures
def _ctx_ok(snap, ctx) -> bool:
    return (type(snap) is dict and all(snap.get(k) == ctx[k] for k in CONTEXT_KEYS)
            and _int(snap.get("process_id"), 1, 2 ** 31 - 1))


def bindings(snapshot, ctx, revision=profiles.BASELINE):
    """(records, reasons, qualification) of one request-id binding snapshot."""
    if type(snapshot) is not dict:
        return [], ["binding_snapshot_missing"], None
    R = []
    src = snapshot.get("source")
    qual = snapshot.get("qualification") if type(snapshot.get("qualification")) is str else None
    if (snapshot.get("schema") != BINDING_SCHEMA or snapshot.get("profile") != profiles.BINDING_PROFILE
            or not _ctx_ok(snapshot, ctx) or snapshot.get("closed") is not True
            or snapshot.get("runtime_qualified") is not False or snapshot.get("release_qualifying") is not False
            or qual not in ("source_bound_candidate", "cpu_source_functions")):
        R.append("binding_snapshot_identity_or_closure_unverified")
    if (type(src) is not dict or src.get("supported") is not True or src.get("profile") != profiles.BINDING_PROFILE
            or src.get("revision") != revision or not ev.same(src.get("files"), profiles.get(revision)["binding_files"])):
        R.append("binding_source_unverified")
    h = snapshot.get("health")
    if (type(h) is not dict or h.get("complete") is not True or h.get("budget_exhausted") is not False
            or any(type(h.get(k)) is not int or h[k] != 0 for k in ("errors", "dropped_records", "late_calls",
                                                                   "active_calls"))):
        R.append("binding_recording_health_unverified")
    recs, bud = snapshot.get("records"), snapshot.get("budgets")
    if type(recs) is not list:
        R.append("binding_record_list_unverified")
        recs = []
    if len(recs) > MAX_REQUESTS:
        raise ev.EvidenceError("binding records exceed the supported bound")
    nbytes = sum(len(ev.json_bytes(r)) for r in recs)
    if (type(bud) is not dict or not _int(bud.get("max_records"), 1, MAX_REQUESTS)
            or not _int(bud.get("max_bytes"), 65536, 8 * 1024 * 1024)
            or type(bud.get("retained_records")) is not int or bud["retained_records"] != len(recs)
            or type(bud.get("retained_bytes")) is not int or bud["retained_bytes"] != nbytes
            or type(bud.get("fixed_metadata_bytes")) is not int or bud["fixed_metadata_bytes"] != BINDING_FIXED_BYTES
            or len(recs) > bud["max_records"] or nbytes + BINDING_FIXED_BYTES > bud["max_bytes"]):
        R.append("binding_snapshot_budget_unverified")
    seqs = [r.get("sequence") if type(r) is dict else None for r in recs]
    if any(not _int(s, 1) for s in seqs) or len(seqs) != len(set(seqs)) or seqs != sorted(seqs):
        R.append("binding_sequence_unverified")
    for r in recs:
        if (type(r) is not dict or not _text(r.get("external_request_id"))
                or r.get("external_req_id") != r.get("external_request_id") or not _text(r.get("internal_request_id"))
                or r.get("randomization_observed") is not True or r.get("native_return_is_none") is not True
                or "engine_exception" not in r or r.get("engine_exception") is not None
                or r.get("external_request_id") == r.get("internal_request_id")):
            R.append("binding_native_assignment_unverified")
        if type(r) is not dict or not _int(r.get("prompt_tokens"), 1, MAX_PROMPT_TOKENS) or not _sha(r.get("prompt_sha256")):
            R.append("native_prompt_recording_unverified")
    return recs, list(dict.fromkeys(R)), qual


def _capture(value, plan, arm) -> dict:
    revision = profiles.get(plan["source_revision"])["revision"]
    ctx = {k: (plan[k] if k in ("run_id", "packet_sha256") else arm[k]) for k in CONTEXT_KEYS}
    if type(value) is not dict:
        return {"issues": ["engine_capture_missing"], "bindings": [], "calls": [], "unverified": [],
                "qualification": "unknown"}
    R = []
    if (any(value.get(k) != ctx[k] for k in ("arm_id", "engine_session_id")) or value.get("source_revision") != revision
            or value.get("capture_complete") is not True):
        R.append("engine_capture_identity_or_closure_unverified")
    st = value.get("startup")
    if (type(st) is not dict or not _sha(value.get("startup_sha256")) or ev.digest(ev.json_bytes(st)) != value.get("startup_sha256")
            or any(st.get(k) != ctx[k] for k in CONTEXT_KEYS) or st.get("source_revision") != revision
            or st.get("role") != "decode" or st.get("model") != plan["model"]
            or not ev.same(st.get("source_profile"), profiles.client_source(revision))
            or st.get("checksum_enabled") is not True or st.get("request_id_randomization_enabled") is not True):
        R.append("engine_startup_binding_unverified")
    bsnaps, csnaps = value.get("binding_snapshots"), value.get("checksum_snapshots")
    if type(bsnaps) is not list:
        R.append("binding_snapshot_list_unverified")
        bsnaps = []
    if type(csnaps) is not list:
        R.append("checksum_snapshot_list_unverified")
        csnaps = []
    if len(bsnaps) > MAX_SNAPSHOTS or len(csnaps) > MAX_SNAPSHOTS:
        raise ev.EvidenceError("capture snapshot lists exceed the supported bound")
    binds, calls, unverified, domains = [], [], [], []
    bact = cact = nrec = 0
    for i, snap in enumerate(bsnaps):
        recs, iss, dom = bindings(snap, ctx, revision)
        R.extend(iss)
        domains.append(dom)
        bact += bool(recs)
        binds.extend({**r, "binding_snapshot_index": i, "process_id": snap.get("process_id")} for r in recs
                     if type(r) is dict)
        if len(binds) > MAX_REQUESTS:
            raise ev.EvidenceError("aggregate binding records exceed the supported bound")
    for i, snap in enumerate(csnaps):
        if type(snap) is dict and type(snap.get("records")) is list:
            nrec += len(snap["records"])
            if nrec > MAX_REQUESTS:
                raise ev.EvidenceError("aggregate checksum records exceed the supported bound")
        if type(snap) is not dict or not _ctx_ok(snap.get("capture_context"), ctx):
            R.append("checksum_capture_context_unverified")
        try:
            rep = observer.snapshot_report(ev.parse_json(ev.json_bytes(snap)), revision=revision)
        except (ev.EvidenceError, TypeError, ValueError) as e:
            R.append("checksum_snapshot_unreadable")
            unverified.append({"request_id": None, "reason": "checksum_snapshot_unreadable", "detail": type(e).__name__})
            continue
        dom = rep["qualification"]
        domains.append(dom if type(dom) is str else None)
        R.extend(x for x in rep["hold_reasons"] if x not in (
            "runtime_qualification_pending", "independent_client_inventory_not_joined",
            "joint_release_profile_not_qualified", "no_recorded_native_verification_calls"))
        cact += bool(snap.get("records"))
        for row in rep["verification_calls"]:
            orig = snap["records"][row["record_index"]]
            proof = orig.get("proof") if type(orig) is dict else None
            cctx = snap.get("capture_context")
            calls.append({**row, "checksum_snapshot_index": i,
                          "checksum_num_tokens": proof.get("num_tokens") if type(proof) is dict else None,
                          "process_id": cctx.get("process_id") if type(cctx) is dict else None})
        unverified.extend(rep["unverified_observations"])
    if bact != 1:
        R.append("unambiguous_active_binding_recorder_missing")
    if cact != 1:
        R.append("unambiguous_active_checksum_recorder_missing")
    if (not domains or any(d not in ("source_bound_candidate", "cpu_source_functions") for d in domains)
            or len(set(domains)) != 1):
        R.append("capture_qualification_domain_unverified")
    return {"issues": list(dict.fromkeys(R)), "bindings": binds, "calls": calls, "unverified": unverified,
            "qualification": domains[0] if domains and len(set(domains)) == 1 else "unknown"}


# ------------------------------------------------------------------------------------------ cache accounting join
def cache_facts(capture, plan, arm) -> dict:
    ctx = {k: plan[k] if k in ("run_id", "packet_sha256") else arm[k] for k in CONTEXT_KEYS}
    out = {}
    for role in ("prefill", "decode"):
        env = capture.get("prefill_capture") if role == "prefill" else capture
        env = env if type(env) is dict else {}
        R, recs, binds = [], [], []
        st = env.get("startup", {})
        st = st if type(st) is dict else {}
        if (st.get("role") != role or any(st.get(k) != v for k, v in ctx.items()) or st.get("prefix_caching") is not True
                or st.get("checksum_enabled") is not True or st.get("source_revision") != plan["source_revision"]
                or not profiles.startup_supported(st, plan["source_revision"])):
            R.append("native_cache_startup_unverified:" + role)
        snaps = env.get("cache_snapshots")
        if type(snaps) is not list or len(snaps) != 1:
            R.append("native_cache_snapshot_missing_or_ambiguous:" + role)
        else:
            recs, errs = observer.cache_snapshot(snaps[0], ctx, role, plan["source_revision"])
            R.extend(errs)
            if type(snaps[0]) is not dict or snaps[0].get("process_id") != st.get("process_id"):
                R.append("native_cache_process_binding_unverified:" + role)
        bs = env.get("binding_snapshots")
        if type(bs) is not list or len(bs) > MAX_SNAPSHOTS:
            R.append("cache_request_binding_snapshots_missing:" + role)
        else:
            active = 0
            for snap in bs:
                rows, errs, dom = bindings(snap, ctx, plan["source_revision"])
                R.extend(errs)
                active += bool(rows)
                binds.extend(rows)
                if snaps and type(snaps) is list and len(snaps) == 1 and type(snaps[0]) is dict:
                    if dom != snaps[0].get("qualification"):
                        R.append("native_cache_qualification_disagrees:" + role)
                if len(binds) > MAX_REQUESTS:
                    raise ev.EvidenceError("native cache bindings exceed their bound")
            if active != 1:
                R.append("cache_request_binding_ambiguous:" + role)
        out[role] = {"records": recs, "bindings": binds, "issues": list(dict.fromkeys(R)), "joined": set()}
    return out


def cache_usage(facts: dict, raw, row: dict, *, for_transfer: bool = False):
    """Per-role cache stats of one request joined through the binding records. Returns (stats by role, issues)."""
    stats, issues = {}, []
    for role in ("prefill", "decode"):
        f = facts[role]
        issues.extend(f["issues"])
        rid = row["prefill_request_id"] if role == "prefill" else row["client_request_id"]
        m = [b for b in f["bindings"] if b.get("external_request_id") == "cmpl-" + rid + "-0"]
        if len(m) != 1:
            issues.append("native_cache_request_join_unverified:" + role)
            continue
        b = m[0]
        internal = b.get("internal_request_id")
        if ((for_transfer and (type(internal) is not str or not internal))
                or sum(x.get("internal_request_id") == internal for x in f["bindings"]) != 1
                or b.get("prompt_sha256") != row["prompt_sha256"]
                or (for_transfer and type(b.get("prompt_tokens")) is not int)
                or b.get("prompt_tokens") != row["prompt_tokens"]
                or (role == "decode" and internal != row.get("internal_request_id"))):
            issues.append("native_cache_request_join_unverified:" + role)
            continue
        f["joined"].add(internal)
        stage = raw.get(role, {}) if type(raw) is dict else {}
        resp = stage.get("response_body", {}) if type(stage) is dict else {}
        resp = resp if type(resp) is dict else {}
        usage = resp.get("usage", {})
        usage = usage if type(usage) is dict else {}
        value, errs = observer.request_usage(f["records"], internal, row["prompt_tokens"], row["prompt_sha256"],
                                             usage.get("completion_tokens"))
        issues.extend(e + ":" + role for e in errs)
        if for_transfer:
            if f["issues"] or errs or type(value) is not dict:
                continue
            if role == "prefill":
                d = resp.get("kv_transfer_params", {})
                if (type(d) is not dict or d.get("remote_request_id") != internal or value["num_external_cached_tokens"] != 0
                        or type(d.get("remote_prefill_cached_tokens")) is not int
                        or d["remote_prefill_cached_tokens"] != value["num_cached_tokens"]):
                    issues.append("producer_cache_descriptor_counts_unverified")
                    continue
            stats[role] = value
            continue
        if not f["issues"] and not errs and type(value) is dict:
            stats[role] = value
        if role == "prefill":
            d = resp.get("kv_transfer_params", {})
            if type(d) is not dict or d.get("remote_request_id") != internal:
                issues.append("producer_cache_transfer_request_binding_unverified")
            if role in stats:
                cached = d.get("remote_prefill_cached_tokens") if type(d) is dict else None
                if stats[role]["num_external_cached_tokens"] != 0 or type(cached) is not int or \
                        cached != stats[role]["num_cached_tokens"]:
                    issues.append("producer_cache_descriptor_counts_unverified")
                    del stats[role]
    return stats, list(dict.fromkeys(issues))


def join_cache(facts, raw, row):
    """Token coverage of one request from cache accounting and its checksum call (full-prompt view)."""
    usage = {"prompt_tokens": row["prompt_tokens"], "transferred_tokens_checked": None,
             "decode_cached_tokens_unchecked": None, "decode_locally_computed_tokens": None,
             "prefill_cached_tokens": None, "prefill_reused_cached_blocks": "unknown"}
    stats, errors = cache_usage(facts, raw, row)
    if "prefill" in stats:
        n = stats["prefill"]["num_local_cached_tokens"]
        usage.update(prefill_cached_tokens=n, prefill_reused_cached_blocks=n > 0)
    if "decode" in stats:
        v = stats["decode"]
        local, remote = v["num_local_cached_tokens"], v["num_external_cached_tokens"]
        usage.update(decode_cached_tokens_unchecked=local, decode_locally_computed_tokens=v["num_computed_tokens"])
        if local:
            errors.append(observer.CACHED_PREFIX_REASON)
        if v["num_computed_tokens"]:
            errors.append("locally_computed_prompt_not_covered_by_checksum")
        calls = row.get("checksum_calls", [])
        scope = calls[0].get("conditional_scope", {}).get("token_coverage", {}) if len(calls) == 1 else {}
        if (len(calls) == 1 and not calls[0].get("recording_issues") and scope.get("prompt_tokens") == row["prompt_tokens"]
                and scope.get("decode_cached_tokens_unchecked") == local and scope.get("transferred_tokens_checked") == remote
                and remote == row["prompt_tokens"] - local):
            usage["transferred_tokens_checked"] = remote
        elif not calls and remote == 0:
            usage["transferred_tokens_checked"] = 0
            errors.append("no_transfer_checksum_comparison_recorded")
        else:
            errors.append("native_cache_to_checksum_span_unverified")
    return usage, list(dict.fromkeys(errors))


def unexpected_cache(facts) -> list[str]:
    out = []
    for role, f in facts.items():
        seen = {r.get("request_id") for r in f["records"] if type(r) is dict and type(r.get("request_id")) is str}
        bound = {r.get("internal_request_id") for r in f["bindings"] if type(r.get("internal_request_id")) is str}
        if seen - f["joined"] or bound - f["joined"]:
            out.append("unexpected_native_cache_requests:" + role)
    return out


# ------------------------------------------------------------------------------------------ the join
def evaluate(plan_raw: bytes, inventory_raw: bytes, captures_raw: bytes) -> dict:
    plan = _read(plan_raw, PLAN_SCHEMA, "checksum request plan")
    inventory = _read(inventory_raw, INVENTORY_SCHEMA, "checksum client inventory")
    captures = _read(captures_raw, CAPTURES_SCHEMA, "checksum client captures")
    planned, arms, _ = planned_rows(plan)
    issues = []
    inv_ok = _bound_to(plan, inventory, plan_raw)
    cap_ok = _bound_to(plan, captures, plan_raw)
    if not inv_ok:
        issues.append("client_inventory_run_binding_unverified")
    if inventory.get("completed") is not True:
        issues.append("client_inventory_completion_unverified")
    if not cap_ok:
        issues.append("capture_manifest_run_binding_unverified")
    raw_rows, raw_caps = inventory.get("requests"), captures.get("captures")
    if type(raw_rows) is not list:
        issues.append("client_inventory_row_list_unverified")
        raw_rows = []
    if len(raw_rows) > MAX_REQUESTS:
        raise ev.EvidenceError("client inventory rows exceed the supported bound")
    if type(raw_caps) is not list:
        issues.append("capture_list_unverified")
        raw_caps = []
    if len(raw_caps) > MAX_ARMS:
        raise ev.EvidenceError("client capture arms exceed the supported bound")
    indexed, unexpected_rows = {}, []
    keys = {(r["arm_id"], r["slot"]) for r in planned}
    for i, raw in enumerate(raw_rows):
        k = (raw.get("arm_id"), raw.get("slot")) if type(raw) is dict else None
        if k is None or type(k[0]) is not str or type(k[1]) is not int or k not in keys:
            unexpected_rows.append({"record_index": i, "reason": "unplanned_or_malformed_client_row"})
        else:
            indexed.setdefault(k, []).append(raw)
    if unexpected_rows:
        issues.append("unexpected_client_inventory_rows")

    def tagged(raw, arm, idx):
        f = _capture(raw, plan, arm)
        for k in ("bindings", "calls", "unverified"):
            f[k] = [{**e, "capture_index": idx} for e in f[k]]
        return f

    by_arm, unexpected_caps, extra = {}, [], []
    for i, raw in enumerate(raw_caps):
        aid = raw.get("arm_id") if type(raw) is dict else None
        if type(aid) is str and aid in arms and arms[aid]["observer_enabled"] is True:
            by_arm.setdefault(aid, []).append((i, raw))
        else:
            unexpected_caps.append({"record_index": i, "reason": "capture_outside_observed_arm"})
            orphan = {"arm_id": aid if _text(aid, 128) else "unknown-capture-" + str(i),
                      "engine_session_id": raw.get("engine_session_id") if type(raw) is dict
                      and _text(raw.get("engine_session_id"), 128) else "unknown-session"}
            f = tagged(raw, orphan, i)
            f["issues"].append("capture_outside_observed_arm")
            extra.append((orphan["arm_id"], f))
    if unexpected_caps:
        issues.append("unexpected_engine_captures")
    arm_facts, cfacts = {}, {}
    for name, arm in arms.items():
        if arm["observer_enabled"] is False:
            arm_facts[name] = {"issues": [], "bindings": [], "calls": [], "unverified": [],
                               "qualification": "observer_disabled"}
            continue
        choices = by_arm.get(name, [])
        parsed = [tagged(raw, arm, i) for i, raw in choices]
        if len(parsed) == 1:
            f = parsed[0]
        elif not parsed:
            f = _capture(None, plan, arm)
        else:
            f = {"issues": list(dict.fromkeys(["ambiguous_engine_captures"] + [x for p in parsed for x in p["issues"]])),
                 "qualification": "unknown", "bindings": [e for p in parsed for e in p["bindings"]],
                 "calls": [e for p in parsed for e in p["calls"]], "unverified": [e for p in parsed for e in p["unverified"]]}
        if not cap_ok:
            f["issues"].append("capture_manifest_run_binding_unverified")
        arm_facts[name] = f
        if plan.get("prefix_caching") is True:
            cfacts[name] = cache_facts(choices[0][1] if len(choices) == 1 else {}, plan, arm)
    all_facts = [(n, f, False) for n, f in arm_facts.items()] + [(n, f, True) for n, f in extra]
    rows, joined_calls, joined_binds = [], set(), set()
    for rq in planned:
        row = dict(rq)
        choices = indexed.get((row["arm_id"], row["slot"]), [])
        raw = choices[0] if len(choices) == 1 else None
        reasons, external = _client_row(raw, row, plan["model"])
        if len(choices) > 1:
            reasons.append("ambiguous_client_receipts")
        if not inv_ok:
            reasons.append("client_inventory_run_binding_unverified")
        row.update(client_status="complete" if not reasons else "unknown", external_request_id=external,
                   internal_request_id=None, binding_status="unknown", native_result="unverified", coverage="unknown",
                   check_status="unverified", checksum_calls=[], unverified_observations=[], reasons=reasons)
        row["token_coverage"] = {"prompt_tokens": row["prompt_tokens"], "transferred_tokens_checked": None,
                                 "decode_cached_tokens_unchecked": None, "decode_locally_computed_tokens": None,
                                 "prefill_cached_tokens": None, "prefill_reused_cached_blocks": "unknown"}
        f = arm_facts[row["arm_id"]]
        if row["observer_enabled"] is False:
            row["binding_status"] = "observer_disabled"
            row["reasons"].append("observer_disabled")
            rows.append(row)
            continue
        row["reasons"].extend(f["issues"])
        bs = [b for b in f["bindings"] if b.get("external_request_id") == external] if external else []
        if len(bs) != 1:
            row["reasons"].append("unambiguous_native_request_binding_missing")
        else:
            b = bs[0]
            internal = b.get("internal_request_id")
            if not _text(internal) or not _int(b.get("sequence"), 1):
                row["reasons"].append("native_request_binding_identity_unverified")
            elif sum(x.get("internal_request_id") == internal for x in f["bindings"]) != 1:
                row["reasons"].append("native_internal_request_binding_ambiguous")
            else:
                row["internal_request_id"] = internal
                if (b.get("prompt_sha256") != row["prompt_sha256"] or type(b.get("prompt_tokens")) is not int
                        or b["prompt_tokens"] != row["prompt_tokens"]):
                    row["reasons"].append("native_prompt_to_client_binding_unverified")
                if row["client_status"] == "complete" and not row["reasons"]:
                    row["binding_status"] = "matched"
                    joined_binds.add((row["arm_id"], b.get("capture_index"), b["binding_snapshot_index"], b["sequence"]))
                row["unverified_observations"] = [e for e in f["unverified"] if e.get("request_id") == internal]
                row["reasons"].extend(e["reason"] for e in row["unverified_observations"] if _text(e.get("reason")))
                calls = [(i, c) for i, c in enumerate(f["calls"]) if c.get("request_id") == internal]
                row["checksum_calls"] = [c for _, c in calls]
                if row["binding_status"] == "matched":
                    for i, _ in calls:
                        joined_calls.add((row["arm_id"], i))
                if len(calls) != 1:
                    row["reasons"].append("unambiguous_native_checksum_call_missing")
                else:
                    c = calls[0][1]
                    row["native_result"] = c["native_result"]
                    if c["coverage"] != "complete":
                        row["reasons"].append(c["engine_pass_not_covered_reason"] or c["reason"])
                    if type(c.get("checksum_num_tokens")) is not int or c["checksum_num_tokens"] != row["prompt_tokens"]:
                        row["reasons"].append("client_prompt_to_checksum_span_unverified")
                    if not row["reasons"] and row["binding_status"] == "matched" and c["coverage"] == "complete":
                        row["coverage"] = "complete"
                        row["check_status"] = "passed" if c["native_result"] == "passed" else "mismatch"
                        if row["check_status"] == "mismatch":
                            row["reasons"].append("native_checksum_mismatch")
        if plan.get("prefix_caching") is True:
            row["token_coverage"], ciss = join_cache(cfacts[row["arm_id"]], raw, row)
            row["reasons"].extend(ciss)
            if ciss:
                tc = row["token_coverage"]
                row["coverage"] = ("partial" if tc["decode_cached_tokens_unchecked"]
                                   and type(tc["transferred_tokens_checked"]) is int and tc["transferred_tokens_checked"] > 0
                                   else "unknown")
                row["check_status"] = "unverified"
        elif len(row["checksum_calls"]) == 1 and not row["checksum_calls"][0].get("recording_issues"):
            row["token_coverage"].update(row["checksum_calls"][0]["conditional_scope"]["token_coverage"])
        if row["native_result"] == "mismatch":
            row["reasons"].append("native_checksum_mismatch")
        row["reasons"] = list(dict.fromkeys(row["reasons"]))
        if not row["checksum_calls"]:
            row["reasons"].append("no_recorded_checksum_call_for_client_request")
        rows.append(row)
    unexpected_calls, unexpected_binds = [], []
    for aid, f, outside in all_facts:
        for b in f["bindings"]:
            s = b.get("sequence")
            k = (aid, b.get("capture_index"), b["binding_snapshot_index"], s) if _int(s, 1) else None
            if outside or k is None or k not in joined_binds:
                unexpected_binds.append({"arm_id": aid, "reason": "native_binding_without_verified_client_join",
                                         "binding": b})
        for i, c in enumerate(f["calls"]):
            if outside or (aid, i) not in joined_calls:
                unexpected_calls.append({"arm_id": aid, "call_index": i,
                                         "reason": "checksum_call_without_verified_client_join", "call": c})
    if unexpected_calls:
        issues.append("unexpected_checksum_calls")
    if unexpected_binds:
        issues.append("unexpected_native_request_bindings")
    for f in cfacts.values():
        issues.extend(unexpected_cache(f))
    complete = sum(r["client_status"] == "complete" for r in rows)
    if not (inv_ok and inventory.get("completed") is True and not unexpected_rows and complete == len(rows)):
        issues.append("client_inventory_incomplete")
    unverified_on = sum(r["observer_enabled"] and r["check_status"] != "passed" for r in rows)
    if unverified_on:
        issues.append("required_checksum_coverage_incomplete")
    summary = {"declared_requests": len(rows), "joined_requests": sum(r["binding_status"] == "matched" for r in rows),
               "checksum_calls": sum(len(f["calls"]) for _, f, _ in all_facts), "joined_checksum_calls": len(joined_calls),
               "native_results": dict(Counter(c["native_result"] for _, f, _ in all_facts for c in f["calls"])),
               "verified_on_requests": sum(r["check_status"] == "passed" for r in rows),
               "on_unverified_requests": unverified_on}
    return {"schema": REPORT_SCHEMA, "source_revision": plan["source_revision"], "summary": summary, "requests": rows,
            "captures": [{"arm_id": n, "qualification": f["qualification"], "issues": f["issues"],
                          "planned_arm": not outside} for n, f, outside in all_facts],
            "hold_reasons": list(dict.fromkeys(issues + list(PROFILE_LIMITS)))}
