"""`sdcguard transfer-check DIR` and `sdcguard transfer-compare BASE CAND`.

transfer-check: a separate obligation from the full-prompt gate. For each request it asks only whether the KV
chunks that actually crossed from prefill to decode (expected units from the receive plan, never from an
intersection with what was compared) were all compared by the native checksum. Statuses VERIFIED, NOT_EXERCISED
(nothing was transferred), MISMATCH, UNOBSERVABLE. The full-prompt verdict is recomputed unchanged. Exit 0 on PASS.

transfer-compare: two recordings of the same workload and configuration on two engine builds; per slot the
transfer coverage is PRESERVED, REGRESSED (a recorded native mismatch after a verified baseline) or UNVERIFIABLE.
Always exits 2: preservation of transfer coverage never overrides the full-prompt HOLD.

The statuses, reason strings and renderings keep the reference's contract (src/sdcguard/transfer_coverage.py:82-304,
transfer_upgrade.py:40-357); the code is this package's own.
"""
from __future__ import annotations

import argparse
import re
import sys
from collections import Counter
from pathlib import Path

from . import client as cl
from . import evidence as ev
from . import gate
from . import observer
from . import profiles

SCHEMA = "sdcguard.transfer-coverage.v1"
SCOPE = "observed native comparison of planned transfer token-chunk positions"
LIMITS = [
    "Only the pinned same-host eager checksum profile with native cache accounting is supported.",
    "Cached decode tokens are outside this transfer obligation and still hold the full-prompt gate.",
    "The checker validates recorded comparison scope and native results, not checksum arrays offline.",
    "Token-chunk positions are not physical bytes, all model layers, ownership or physical reads.",
    "Cross-machine correctness and runtime qualification remain unknown.",
    "Input hashes show local consistency, not execution attestation or recorder authenticity.",
]
OWNER = gate.OWNER


def _uniq(xs):
    return list(dict.fromkeys(xs))


def _int(v, lo=0, hi=cl.MAX_PROMPT_TOKENS):
    return type(v) is int and lo <= v <= hi


def transfer_scope(plans, records, *, prompt_tokens, local_tokens, remote_tokens) -> dict:
    """Expected transfer chunks from the receive plan, compared chunks from the verification record."""
    res = dict(status="UNOBSERVABLE", reasons=[], expected_units=None, compared_units=None,
               expected_tokens=remote_tokens, compared_tokens=None, native_result="unverified", plan_sequence=None,
               update_sequence=None, verification_sequence=None)
    R = res["reasons"]
    if (not _int(prompt_tokens, 1) or not _int(local_tokens) or not _int(remote_tokens)
            or local_tokens + remote_tokens != prompt_tokens):
        R.append("native_transfer_token_accounting_unverified")
        return res
    if remote_tokens == 0:
        if plans or records:
            R.append("zero_transfer_has_checksum_activity")
        else:
            res.update(status="NOT_EXERCISED", expected_units=[], compared_units=[], compared_tokens=0)
        return res
    if len(plans) != 1 or len(records) != 1 or records[0].get("kind") != "verification":
        R.append("transfer_plan_or_verification_missing_or_ambiguous")
        return res
    plan, rec = plans[0], records[0]
    load, proof = plan.get("load_plan"), rec.get("proof")
    if type(load) is not dict or type(proof) is not dict:
        R.append("transfer_plan_metadata_missing")
        return res
    pid, pev = plan.get("plan_sequence"), plan.get("sequence")
    upd, ver = rec.get("origin_update_sequence"), rec.get("sequence")
    res.update(plan_sequence=pid, update_sequence=upd, verification_sequence=ver)
    if (any(not _int(n, 1, 2 ** 63 - 1) for n in (pid, pev, upd, ver)) or not pid < pev < upd < ver
            or type(proof.get("plan_sequence")) is not int or proof["plan_sequence"] != pid
            or not plan.get("request_id") or plan.get("request_id") != rec.get("request_id")):
        R.append("receive_plan_to_verification_join_unverified")
    if not observer.plan_matches_proof(plan, proof):
        R.append("planned_chunk_scope_disagrees_with_verification")
    if (type(load.get("num_tokens")) is not int or load["num_tokens"] != prompt_tokens
            or type(load.get("num_local_computed_tokens")) is not int or load["num_local_computed_tokens"] != local_tokens):
        R.append("receive_plan_disagrees_with_native_cache_accounting")
    groups = load.get("groups")
    if type(groups) is not list or len(groups) != 1 or type(groups[0]) is not dict:
        R.append("transfer_group_layout_unsupported")
    else:
        g = groups[0]
        gid, size, start, count = (g.get(k) for k in ("group_id", "block_size", "start", "block_count"))
        if (not _int(gid) or not _int(size, 1) or not _int(start) or not _int(count, 1, observer.MAX_UNITS)
                or local_tokens % size or start != local_tokens // size
                or count != (prompt_tokens + size - 1) // size - start):
            R.append("receive_plan_does_not_cover_transfer_span")
        else:
            res["expected_units"] = [f"group:{gid}:chunk:{n}" for n in range(start, start + count)]
    d = observer.classify_verification(rec, max_units=observer.MAX_UNITS)
    R.extend(r for r in d["reasons"] if r != observer.CACHED_PREFIX_REASON)
    res.update(native_result=d["native_result"], compared_units=d["compared_units"])
    if not res["expected_units"] or res["compared_units"] != res["expected_units"]:
        R.append("transfer_comparison_scope_incomplete")
    if d["native_result"] == "mismatch":
        R.append("native_checksum_mismatch")
    elif d["native_result"] != "passed" or rec.get("native_return") is not True:
        R.append("native_passing_checksum_not_recorded")
    res["reasons"] = _uniq(R)
    if not R:
        res.update(status="VERIFIED", compared_tokens=remote_tokens)
    elif d["native_result"] == "mismatch":
        res["status"] = "MISMATCH"
    return res


def evaluate(result_raw, archive_raw, preflight_raw) -> dict:
    full = gate.checksum_gate(result_raw, archive_raw, preflight_raw, ["checksum"])
    issues = [r for r in full["hold_reasons"] if r != gate.COVERAGE_HOLD]
    files = ev.read_archive(archive_raw)
    plan = ev.object_at(files, "client/REQUEST_PLAN.json")
    inventory = ev.object_at(files, "client/CLIENT_INVENTORY.json")
    captures = ev.object_at(files, "CAPTURES.json")["captures"]
    joined = cl.evaluate(files["client/REQUEST_PLAN.json"], files["client/CLIENT_INVENTORY.json"], files["CAPTURES.json"])
    if plan.get("prefix_caching") is not True:
        issues.append("transfer_profile_requires_native_cache_accounting")
    cfacts = {}
    for arm in plan["arms"]:
        m = [c for c in captures if c.get("arm_id") == arm["arm_id"]]
        if arm["observer_enabled"] and len(m) == 1 and plan.get("prefix_caching") is True:
            cfacts[arm["arm_id"]] = cl.cache_facts(m[0], plan, arm)
    known = {(r["arm_id"], r["internal_request_id"]) for r in joined["requests"] if type(r["internal_request_id"]) is str}
    for cap in captures:
        for snap in cap.get("checksum_snapshots", []):
            for rec in snap.get("records", []):
                if type(rec) is not dict or (cap["arm_id"], rec.get("request_id")) not in known:
                    issues.append("unjoined_native_transfer_record")
    rows = []
    for row in joined["requests"]:
        errors, acct = [], {}
        if row["client_status"] != "complete":
            errors.append("client_request_completion_unverified")
        if row["binding_status"] != "matched":
            errors.append("client_to_native_request_join_unverified")
        if not row["observer_enabled"]:
            errors.append("observer_disabled")
        raws = [r for r in inventory["requests"] if type(r) is dict and r.get("arm_id") == row["arm_id"]
                and r.get("slot") == row["slot"]]
        f = cfacts.get(row["arm_id"])
        if f is None or len(raws) != 1:
            errors.append("native_cache_accounting_unavailable")
        else:
            acct, cerr = cl.cache_usage(f, raws[0], row, for_transfer=True)
            errors.extend(cerr)
        sel = [c for c in captures if c.get("arm_id") == row["arm_id"]]
        snaps = sel[0].get("checksum_snapshots", []) if len(sel) == 1 else []
        recs = [r for s in snaps for r in s.get("records", []) if type(r) is dict
                and type(row["internal_request_id"]) is str and r.get("request_id") == row["internal_request_id"]]
        plans = [r for r in recs if r.get("kind") == "recv_plan"]
        other = [r for r in recs if r.get("kind") != "recv_plan"]
        dec, pre = acct.get("decode", {}), acct.get("prefill", {})
        local, remote = dec.get("num_local_cached_tokens"), dec.get("num_external_cached_tokens")
        scoped = transfer_scope(plans, other, prompt_tokens=row["prompt_tokens"], local_tokens=local,
                                remote_tokens=remote)
        if dec.get("num_computed_tokens") != 0:
            errors.append("locally_computed_prompt_scope_unsupported")
        if len(acct) != 2:
            errors.append("both_native_cache_accounts_required")
        for call in row["checksum_calls"]:
            errors.extend(call["recording_issues"])
        for cap in joined["captures"]:
            if cap["arm_id"] == row["arm_id"]:
                errors.extend(cap["issues"])
        status = scoped["status"]
        empty_ok = {"unambiguous_active_checksum_recorder_missing", "client_to_native_request_join_unverified"}
        if errors and (status != "NOT_EXERCISED" or set(errors) - empty_ok):
            status = "UNOBSERVABLE"
        rows.append(dict(client_request_id=row["client_request_id"], arm_id=row["arm_id"], slot=row["slot"],
                         internal_request_id=row["internal_request_id"], status=status,
                         reasons=_uniq(errors + scoped["reasons"]), comparison=scoped,
                         tokens=dict(prompt=row["prompt_tokens"], expected_transfer=remote,
                                     compared_transfer=scoped["compared_tokens"] if not errors else None,
                                     decode_cache_outside_transfer=local,
                                     prefill_cache_reused=pre.get("num_local_cached_tokens"))))
    for f in cfacts.values():
        issues.extend(cl.unexpected_cache(f))
    issues = _uniq(issues)
    for row in rows:
        row["reasons"] = _uniq(row["reasons"] + issues)
        row["decision"] = "HOLD" if row["reasons"] or row["status"] not in ("VERIFIED", "NOT_EXERCISED") else (
            "NOT_EXERCISED" if row["status"] == "NOT_EXERCISED" else "PASS")
    counts = Counter(r["status"] for r in rows)
    if not rows or not counts["VERIFIED"]:
        issues.append("no_verified_transfer_requests")
    if any(r["decision"] == "HOLD" for r in rows):
        issues.append("transfer_comparison_obligation_incomplete")

    def total(name):
        vals = [r["tokens"][name] for r in rows]
        return sum(vals) if vals and all(type(v) is int for v in vals) else None
    exp = [r["comparison"]["expected_units"] for r in rows]
    exp_n = sum(len(u) for u in exp) if exp and all(type(u) is list for u in exp) else None
    return dict(schema=SCHEMA, owner=OWNER, scope=SCOPE, transfer_decision="HOLD" if issues else "PASS",
                release_decision=full["decision"], full_prompt_gate=full, runtime_qualified=False, engine=full["engine"],
                inputs_sha256=dict(result=ev.digest(result_raw), archive=ev.digest(archive_raw),
                                   preflight=ev.digest(preflight_raw) if preflight_raw is not None else None),
                summary=dict(planned_requests=len(rows), verified_requests=sum(r["decision"] == "PASS" for r in rows),
                             not_exercised_requests=counts["NOT_EXERCISED"],
                             held_requests=sum(r["decision"] == "HOLD" for r in rows), statuses=dict(counts),
                             expected_chunk_positions=exp_n, prompt_tokens=total("prompt"),
                             expected_transfer_tokens=total("expected_transfer"),
                             compared_transfer_tokens=total("compared_transfer"),
                             decode_cached_tokens_outside_transfer=total("decode_cache_outside_transfer")),
                hold_reasons=_uniq(issues), requests=rows, limits=LIMITS)


def _read_dir(path: Path) -> dict:
    names = ["RESULT.json", "ordinary-evidence.zip"]
    if (path / "CPU_PREFLIGHT.json").exists():
        names.append("CPU_PREFLIGHT.json")
    return {n: ev.read_file(path, n) for n in names}


def inspect(path) -> dict:
    path = Path(path)
    raw = _read_dir(path)
    ans = evaluate(raw["RESULT.json"], raw["ordinary-evidence.zip"], raw.get("CPU_PREFLIGHT.json"))
    if _read_dir(path) != raw:
        raise ev.EvidenceError("owner inputs changed during inspection")
    return ans


def render(ans: dict) -> str:
    lines = ["Transfer comparison: " + ans["transfer_decision"], "Full-prompt policy: " + ans["release_decision"], SCOPE]
    if "summary" in ans:
        s = ans["summary"]
        lines.append(f"{s['verified_requests']} / {s['planned_requests']} requests verified for this transfer obligation")
        lines.append(f"Transferred tokens compared: {s['compared_transfer_tokens']}; decode-cache tokens outside "
                     f"transfer: {s['decode_cached_tokens_outside_transfer']}")
    lines.extend("HOLD: " + r for r in ans["hold_reasons"])
    for row in ans.get("requests", []):
        t = row["tokens"]
        lines.append(f"{row['client_request_id']} | {row['status']} | {row['decision']} | "
                     + ("; ".join(row["reasons"]) or "complete recorded transfer comparison"))
        lines.append(f"  transfer tokens: {t['compared_transfer']} / {t['expected_transfer']}; cached outside transfer: "
                     f"{t['decode_cache_outside_transfer']}")
    lines.extend(ans["limits"])
    return "\n".join(lines) + "\n"


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="sdcguard transfer-check", description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("input", help="saved owner-result directory; no runtime execution")
    ap.add_argument("--json", action="store_true")
    a = ap.parse_args(argv)
    try:
        ans = inspect(a.input)
    except (ValueError, OSError, KeyError, TypeError, AttributeError, IndexError) as e:
        ans = dict(schema=SCHEMA, transfer_decision="HOLD", release_decision="HOLD",
                   hold_reasons=["evidence_unverifiable:" + str(e)], limits=LIMITS)
    sys.stdout.write(ev.json_bytes(ans).decode() if a.json else render(ans))
    return 0 if ans["transfer_decision"] == "PASS" else 2


# ================================================================================== transfer-compare
UP_SCHEMA = "sdcguard.transfer-upgrade.v1"
POLICY = "preserve-recorded-transfer-coverage.v1"
ERRORS = (ValueError, OSError, KeyError, TypeError, AttributeError, IndexError)
UP_LIMITS = [
    "Changes describe recorded coverage, not a cause or an engine correctness failure.",
    "Only matching workloads and recorded configuration can support coverage preservation.",
    "Missing evidence is UNVERIFIABLE; REGRESSED requires a recorded native mismatch after a verified baseline.",
    "Identical inputs, different paths, run IDs or packet hashes do not prove independent builds.",
    "Only the two exact recorded checksum source profiles are supported.",
    "Transfer preservation is separate from the full-prompt release decision, which remains HOLD.",
    "Input hashes establish local consistency, not execution or recorder authenticity.",
    "Full-prompt release decisions are recomputed unchanged. Cached tokens remain outside transfer scope.",
]
_STARTUP_VOLATILE = {"run_id", "packet_sha256", "engine_session_id", "process_id", "actual_model", "actual_tokenizer",
                     "snapshot", "source_revision", "source_identity", "source_profile", "native_transport"}
_REQUIRED_CONFIG = {"model", "model_revision", "prefix_caching", "checksum_enabled", "parallel", "dtype", "kv_dtype",
                    "block_size", "group_specs", "gpu_blocks", "max_model_len", "max_num_seqs", "connector", "role",
                    "transfer_role", "transfer_extra", "transport_profile", "model_runner_v2", "async_scheduling",
                    "chunked_prefill", "speculative_disabled", "flashinfer_sampler_enabled", "multiprocess_method",
                    "request_id_randomization_enabled"}
_TRANSFER_VOLATILE = {"remote_request_id", "remote_block_ids", "remote_engine_id", "remote_host", "remote_port",
                      "remote_blocks_expiry_time", "remote_registration_generation", "remote_prefill_cached_tokens",
                      "remote_num_tokens", "kv_checksums"}


def _h(v) -> str:
    return ev.digest(ev.json_bytes(v))


def _without(v, names):
    if type(v) is not dict:
        raise ev.EvidenceError("comparison metadata must be an object")
    return {k: x for k, x in v.items() if k not in names}


def _key(row):
    a, s = row["arm_id"], row["slot"]
    if type(a) is not str or not a or type(s) is not int or s < 0:
        raise ev.EvidenceError("invalid comparison slot")
    return a, s


def _index(rows):
    out = {}
    for r in rows:
        k = _key(r)
        if k in out:
            raise ev.EvidenceError("duplicate comparison slot")
        out[k] = r
    return out


def _engine_identity(pre):
    inst = pre["installed_engine"]
    out = {k: inst[k] for k in ("source_revision", "source_files", "compiled_members")}
    out["extracted_members"] = inst["precompiled_payload"]["extracted_members"]
    if not all(out[k] for k in out):
        raise ev.EvidenceError("engine identity is incomplete")
    return out


def _runtime_identity(pre):
    inst = pre["installed_engine"]
    py, vers = inst["python_identity"], inst["versions"]
    ver = py.get("version")
    if (type(vers) is not dict or not {"vllm", "torch", "triton", "nixl", "nixl-cu12", "nixl-cu13"} <= vers.keys()
            or any(type(v) is not str or re.fullmatch(r"[0-9][0-9A-Za-z.+_-]{0,127}", v) is None
                   for k, v in vers.items() if k != "uv")
            or py.get("implementation") != "cpython" or py.get("platform") != "linux"
            or py.get("soabi") != "cpython-312-x86_64-linux-gnu" or type(ver) is not list or len(ver) != 3
            or any(type(n) is not int or not 0 <= n <= 999 for n in ver) or ver[:2] != [3, 12]):
        raise ev.EvidenceError("recorded runtime identity is missing, unknown or unsupported")
    return dict(versions={k: v for k, v in vers.items() if k != "uv"},
                python={k: py[k] for k in ("implementation", "version", "platform", "soabi")})


def _contracts(files, pre) -> dict:
    plan = ev.object_at(files, "client/REQUEST_PLAN.json")
    inv = ev.object_at(files, "client/CLIENT_INVENTORY.json")
    caps = ev.object_at(files, "CAPTURES.json")["captures"]
    raw_rows = _index(inv["requests"])
    work = _without(plan, {"run_id", "packet_sha256", "source_revision", "arms"})
    work["arms"] = []
    slots, sessions, configs = {}, [], []
    for arm in plan["arms"]:
        norm = _without(arm, {"engine_session_id", "requests"})
        norm["requests"] = []
        for r in arm["requests"]:
            k = _key(dict(arm_id=arm["arm_id"], slot=r["slot"]))
            if k in slots:
                raise ev.EvidenceError("duplicate planned comparison slot")
            spec = _without(r, {"client_request_id", "prefill_request_id"})
            spec["client_inputs"] = {}
            raw = raw_rows.get(k)
            if raw is None:
                raise ev.EvidenceError("client input missing from comparison slot")
            for role in ("prefill", "decode"):
                st = raw[role]
                body = _without(st["request_body"], {"request_id", "kv_transfer_params"})
                body["kv_transfer_params"] = _without(st["request_body"]["kv_transfer_params"], _TRANSFER_VOLATILE)
                hdrs = _without(st["request_headers"], {"X-Request-Id"})
                spec["client_inputs"][role] = dict(method=st["method"], path=st["path"], body_sha256=_h(body),
                                                   headers_sha256=_h(hdrs))
            slots[k] = _h(spec)
            norm["requests"].append(spec)
        work["arms"].append(norm)
    if set(raw_rows) != set(slots):
        raise ev.EvidenceError("client inventory and planned comparison slots differ")
    for cap in caps:
        sess = cap["engine_session_id"]
        if type(sess) is not str or not sess:
            raise ev.EvidenceError("engine session missing")
        sessions.append(sess)
        for role, v in (("decode", cap), ("prefill", cap["prefill_capture"])):
            st = v["startup"]
            if not _REQUIRED_CONFIG <= st.keys():
                raise ev.EvidenceError("recorded comparison configuration is incomplete")
            cfg = _without(st, _STARTUP_VOLATILE)
            if plan["source_revision"] == profiles.BASELINE and cfg.get("defer_async_loads") == "not_in_source_profile":
                cfg["defer_async_loads"] = False
            configs.append(dict(arm_id=cap["arm_id"], role=role, config=cfg))
    model = pre["model_cache"]
    if not all(model.get(k) for k in ("model", "revision", "files")):
        raise ev.EvidenceError("model and tokenizer file identities are missing")
    rt = _runtime_identity(pre)
    rt["versions"].pop("vllm")
    conf = dict(engines=configs, model={k: model[k] for k in ("model", "revision", "files")}, runtime=rt)
    return dict(workload_sha256=_h(work), config_sha256=_h(conf), slots=slots, sessions=sorted(sessions),
                run_id=plan["run_id"])


def _side(raw) -> dict:
    hashes = {k: ev.digest(v) if v is not None else None for k, v in zip(("result", "archive", "preflight"), raw)}
    side = dict(inputs_sha256=hashes, errors=[], assessment=None, contracts=None, engine_identity_sha256=None)
    try:
        side["assessment"] = evaluate(*raw)
        files = ev.read_archive(raw[1])
        pre = ev.parse_json(raw[2]) if raw[2] is not None else {}
        side["contracts"] = _contracts(files, pre)
        gaps = [r for r in side["assessment"]["hold_reasons"] if r not in {
            "required_checksum_coverage_incomplete", "transfer_comparison_obligation_incomplete",
            "no_verified_transfer_requests"}]
        side["errors"].extend("input_qualification:" + r for r in gaps)
        if not gaps:
            side["engine_identity_sha256"] = _h(_engine_identity(pre))
    except ERRORS as e:
        side["errors"].append("evidence_unverifiable:" + str(e))
    return side


def _view(side):
    a, c = side["assessment"], side["contracts"]
    return dict(inputs_sha256=side["inputs_sha256"], errors=side["errors"], engine=a["engine"] if a else None,
                engine_identity_sha256=side["engine_identity_sha256"],
                recording={k: c[k] for k in ("run_id", "sessions")} if c else None,
                workload_sha256=c["workload_sha256"] if c else None, config_sha256=c["config_sha256"] if c else None,
                transfer_decision=a["transfer_decision"] if a else "HOLD",
                full_prompt_gate=a["full_prompt_gate"] if a else None, summary=a["summary"] if a else None,
                hold_reasons=a["hold_reasons"] if a else side["errors"])


def _row_view(row):
    if row is None:
        return None
    return dict({k: row[k] for k in ("client_request_id", "status", "decision", "reasons", "tokens")},
                expected_chunk_positions=row["comparison"]["expected_units"],
                compared_chunk_positions=row["comparison"]["compared_units"])


def _change(before, after, comparable, same_slot):
    if not comparable or not same_slot:
        return "UNVERIFIABLE", ["workload_or_configuration_not_comparable"]
    if before is None or after is None:
        return "UNVERIFIABLE", ["request_missing_from_one_side"]
    if before["decision"] != "PASS":
        return "UNVERIFIABLE", ["baseline_transfer_not_verified"]
    b, a = before["tokens"], after["tokens"]
    keys = ("prompt", "expected_transfer", "decode_cache_outside_transfer", "prefill_cache_reused")
    if (any(type(t[k]) is not int for t in (b, a) for k in keys)
            or any(type(r["comparison"]["expected_units"]) is not list or not r["comparison"]["expected_units"]
                   for r in (before, after))):
        return "UNVERIFIABLE", ["transfer_scope_unverifiable"]
    if any(b[k] != a[k] for k in keys) or before["comparison"]["expected_units"] != after["comparison"]["expected_units"]:
        return "UNVERIFIABLE", ["transfer_exercise_changed"]
    if after["decision"] != "PASS":
        c = after["comparison"]
        if (after["status"] == "MISMATCH" and c["native_result"] == "mismatch"
                and set(after["reasons"]) == {"native_checksum_mismatch"} and set(c["reasons"]) == {"native_checksum_mismatch"}
                and c["compared_units"] == c["expected_units"]):
            return "REGRESSED", ["candidate_recorded_native_mismatch"]
        return "UNVERIFIABLE", ["candidate_transfer_evidence_unverifiable"]
    return "PRESERVED", []


def compare(baseline_raw, candidate_raw) -> dict:
    base, cand = _side(baseline_raw), _side(candidate_raw)
    b, c = base["contracts"], cand["contracts"]
    errors = [f"{lab}:{e}" for lab, s in (("baseline", base), ("candidate", cand)) for e in s["errors"]]
    if not (b is not None and c is not None and b["workload_sha256"] == c["workload_sha256"]):
        errors.append("workload_not_comparable")
    if not (b is not None and c is not None and b["config_sha256"] == c["config_sha256"]):
        errors.append("configuration_not_comparable")
    comparable = not errors
    bi, ci = base["engine_identity_sha256"], cand["engine_identity_sha256"]
    build = "unknown" if bi is None or ci is None else ("same_recorded_build" if bi == ci else "different_recorded_build")
    relation = "unknown"
    if base["inputs_sha256"] == cand["inputs_sha256"]:
        relation = "same_evidence"
    elif b is not None and c is not None and not base["errors"] and not cand["errors"]:
        relation = ("distinct_recorded_sessions" if b["run_id"] != c["run_id"] and not set(b["sessions"]) & set(c["sessions"])
                    else "overlapping_recording_identity")
    before = _index(base["assessment"]["requests"]) if base["assessment"] else {}
    after = _index(cand["assessment"]["requests"]) if cand["assessment"] else {}
    rows = []
    for k in sorted(before.keys() | after.keys()):
        left, right = before.get(k), after.get(k)
        same_slot = b is not None and c is not None and k in b["slots"] and b["slots"].get(k) == c["slots"].get(k)
        st, why = _change(left, right, comparable, same_slot)
        rows.append(dict(arm_id=k[0], slot=k[1], coverage_change=st, reasons=why,
                         lost_passing_evidence=bool(left and left["decision"] == "PASS" and (
                             not right or right["decision"] != "PASS")),
                         baseline=_row_view(left), candidate=_row_view(right)))
    counts = Counter(r["coverage_change"] for r in rows)
    holds = list(errors)
    if counts["REGRESSED"]:
        holds.append("recorded_native_comparison_regressed")
    if counts["UNVERIFIABLE"] or not rows:
        holds.append("coverage_preservation_unverifiable")
    if relation != "distinct_recorded_sessions":
        holds.append("independent_recordings_not_established")
    if build != "different_recorded_build":
        holds.append("changed_engine_build_not_established")
    for lab, s in (("baseline", base), ("candidate", cand)):
        a = s["assessment"]
        if a is None or a["transfer_decision"] != "PASS":
            holds.append(lab + "_transfer_check_held")
        if a is None or a["release_decision"] != "PASS":
            holds.append(lab + "_full_prompt_policy_held")
    pair = tuple(s["assessment"]["engine"].get("source_revision") if s["assessment"] else None for s in (base, cand))
    transition = pair == (profiles.BASELINE, profiles.CANDIDATE) and comparable
    preserved = (transition and relation == "distinct_recorded_sessions" and build == "different_recorded_build" and rows
                 and counts["PRESERVED"] == len(rows)
                 and all(s["assessment"]["transfer_decision"] == "PASS" for s in (base, cand)))
    if not transition:
        holds.append("changed_build_transition_not_qualified")
    return dict(schema=UP_SCHEMA, owner=OWNER, policy=POLICY, scope=SCOPE, upgrade_decision="HOLD",
                transfer_preservation_decision="PASS" if preserved else "HOLD",
                runtime_upgrade_witness="distinct source-bound recordings" if preserved else "not established",
                comparison_status="COMPARABLE" if comparable else "UNVERIFIABLE", build_relation=build,
                recording_relation=relation,
                summary=dict(compared_slots=len(rows), preserved=counts["PRESERVED"], regressed=counts["REGRESSED"],
                             unverifiable=counts["UNVERIFIABLE"],
                             lost_passing_evidence=sum(r["lost_passing_evidence"] for r in rows)),
                baseline=_view(base), candidate=_view(cand), requests=rows, hold_reasons=list(dict.fromkeys(holds)),
                limits=UP_LIMITS)


def inspect_pair(baseline, candidate) -> dict:
    paths = (Path(baseline), Path(candidate))
    raw = [_read_dir(p) for p in paths]
    ans = compare(*(tuple(x.get(n) for n in ("RESULT.json", "ordinary-evidence.zip", "CPU_PREFLIGHT.json")) for x in raw))
    if any(_read_dir(p) != x for p, x in zip(paths, raw)):
        raise ev.EvidenceError("comparison inputs changed during inspection")
    return ans


def render_compare(ans: dict) -> str:
    lines = ["Offline upgrade comparison: " + ans["upgrade_decision"],
             "Transfer preservation: " + ans.get("transfer_preservation_decision", "HOLD")]
    if "summary" in ans:
        s = ans["summary"]
        lines.extend(["Recorded builds: " + ans["build_relation"], "Recordings: " + ans["recording_relation"],
                      f"Coverage: {s['preserved']} preserved, {s['regressed']} regressed, {s['unverifiable']} unverifiable",
                      "Runtime upgrade witness: " + ans["runtime_upgrade_witness"]])
        for lab in ("baseline", "candidate"):
            side = ans[lab]
            full = side["full_prompt_gate"]
            lines.append(f"{lab}: transfer {side['transfer_decision']}; full-prompt {full['decision'] if full else 'HOLD'}")
        for row in ans["requests"]:
            if row["coverage_change"] != "PRESERVED":
                lines.append(f"{row['arm_id']} slot {row['slot']}: {row['coverage_change']} | " + "; ".join(row["reasons"]))
                for lab in ("baseline", "candidate"):
                    v = row[lab]
                    if v:
                        lines.append(f"  {lab} {v['client_request_id']}: {v['decision']} | " + "; ".join(v["reasons"]))
    lines.extend("HOLD: " + r for r in ans["hold_reasons"])
    lines.extend(UP_LIMITS)
    return "\n".join(lines) + "\n"


def main_compare(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="sdcguard transfer-compare", description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("baseline", help="retained baseline owner-result directory")
    ap.add_argument("candidate", help="retained candidate owner-result directory")
    ap.add_argument("--json", action="store_true")
    a = ap.parse_args(argv)
    try:
        ans = inspect_pair(a.baseline, a.candidate)
        out = ev.json_bytes(ans).decode() if a.json else render_compare(ans)
    except ERRORS as e:
        ans = dict(schema=UP_SCHEMA, upgrade_decision="HOLD", hold_reasons=["evidence_unverifiable:" + str(e)],
                   limits=UP_LIMITS)
        out = ev.json_bytes(ans).decode() if a.json else render_compare(ans)
    sys.stdout.write(out)
    return 2
