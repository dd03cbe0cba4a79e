"""`sdcguard gate DIR --require checksum`: offline per-request coverage gate over a recorded prefill/decode run.

PASS applies to the selected recorded requests and check only: a request passes when the native KV checksum
compared its whole prompt and every piece of evidence that binds the comparison to that request is intact.
Anything unverifiable holds. Exit 0 on PASS, 2 on HOLD. Nothing is executed and no device is used.

Inputs (a recorded owner-result directory): RESULT.json, ordinary-evidence.zip (request plan, client inventory and
journal, engine captures, close receipts, cleanup evidence) and CPU_PREFLIGHT.json (engine build identity).

Verdict rules, reason strings and the text rendering keep the reference's contract (src/sdcguard/required_gate.py:
68-490, native_checks.py:54-93) so that saved recordings give the same verdicts; the code is this package's own.
Engine-build attestation of the reference's vLLM recorder is checked for internal consistency (witness and digests);
the reference additionally re-hashes its own installed files and pinned build artifacts, which are not part of a
recording.
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

from . import client as cl
from . import evidence as ev
from . import profiles

CHECKS = ("lease", "checksum")
CONTEXT = ("run_id", "packet_sha256", "arm_id", "engine_session_id")
NATIVE_RESULTS = ("passed", "mismatch", "unverified", "not_compared")
SCOPE = "selected recorded client requests only; no deployment or isolation guarantee"
OWNER = "Hari Krishna Kancharla"     # the verdict schema names the owner of the recorded-evidence format
MODEL = "Qwen/Qwen3-0.6B"
MODEL_REVISION = "c1899de289a04d12100db370d81485cdf75e47ca"
INSTALLED_SCHEMA = "sdcguard.installed-checksum-preflight.v1"
INSTALLED_WITNESS = "sdcguard.installed-checksum-witness.v1"
COVERAGE_HOLD = "required_checksum_coverage_incomplete"


# ------------------------------------------------------------------------------------------ per-check policy
def _units(v, name):
    if v is None:
        return None
    if type(v) is not list or any(type(u) is not str or not u for u in v) or len(set(v)) != len(v):
        raise ValueError(name + " must be unique non-empty strings")
    return list(v)


def assess_check(check_id, *, native_result, expected_units, compared_units, completed, evidence_complete,
                 applicable=True, reason=None) -> dict:
    """Status of one check from normalised facts: passed only with a passing native result, completed call,
    complete evidence and complete coverage of the eligible units."""
    if check_id not in CHECKS or native_result not in NATIVE_RESULTS:
        raise ValueError("unsupported check or native result")
    if (type(completed) is not bool or type(evidence_complete) is not bool
            or (applicable is not None and type(applicable) is not bool)
            or (reason is not None and (type(reason) is not str or not reason or len(reason) > 1024))):
        raise ValueError("explicit boolean completion and bounded reason are required")
    exp, cmp_ = _units(expected_units, "expected_units"), _units(compared_units, "compared_units")
    if exp is not None and cmp_ is not None and not set(cmp_) <= set(exp):
        raise ValueError("compared units include units outside the eligible scope")
    missing = sorted(set(exp or ()) - set(cmp_ or ())) if exp is not None else None
    coverage = ("unknown" if exp is None or cmp_ is None or not evidence_complete
                else "not_covered" if not exp or not cmp_ or applicable is False
                else "partial" if missing else "complete")
    status, why = "unverified", reason
    if applicable is not True:
        why = why or ("not_applicable" if applicable is False else "applicability_unknown")
    elif native_result == "mismatch" and evidence_complete and completed and cmp_:
        status, why = "mismatch", why or "recorded_native_mismatch"
    elif native_result == "passed" and completed and evidence_complete and coverage == "complete":
        status, why = "passed", reason or "complete_recorded_comparison"
    else:
        why = why or ("recording_incomplete" if not evidence_complete else
                      "expected_scope_unknown" if exp is None else
                      "no_eligible_comparison_units" if not exp else
                      "comparison_scope_partial" if coverage == "partial" else
                      "no_recorded_comparison" if not cmp_ else
                      "comparison_not_completed" if not completed else "no_recorded_passing_result")
    return {"check": check_id, "native_result": native_result, "check_status": status, "coverage": coverage,
            "coverage_complete": coverage == "complete", "expected_units": exp, "compared_units": cmp_,
            "missing_units": missing, "completed": completed, "evidence_complete": evidence_complete,
            "applicable": applicable, "reason": why}


def decide(requests, required, issues=(), *, total=None, engine=None, arm=None) -> dict:
    """Apply the required-check policy to per-request facts; supplied statuses are never trusted."""
    if not required or any(c not in CHECKS for c in required) or len(set(required)) != len(required):
        raise ev.EvidenceError("require lease, checksum, or both once each")
    holds = list(issues)
    if len(required) != 1:
        holds.append("combined_lease_checksum_not_supported")
    if not requests:
        holds.append("no_verified_request_denominator")
    rows = []
    for rq in requests:
        reasons = list(rq.get("reasons", []))
        for name in required:
            item = rq.get("checks", {}).get(name)
            if type(item) is not dict:
                reasons.append(name + ":not_recorded")
                continue
            if item.get("check", name) != name:
                reasons.append(name + ":different_check_recorded")
                continue
            a = assess_check(name, native_result=item.get("native_result", "unverified"),
                             expected_units=item.get("expected_units"), compared_units=item.get("compared_units"),
                             completed=item.get("completed") is True, evidence_complete=item.get("evidence_complete") is True,
                             applicable=item.get("applicable"), reason=item.get("reason"))
            if a["check_status"] != "passed":
                reasons.append(name + ":" + a["reason"])
        every = list(dict.fromkeys(reasons + holds))
        rows.append(dict(rq, decision="HOLD" if every else "PASS", reasons=every))
    failed = [r for r in rows if r["decision"] == "HOLD"]
    return dict(schema="sdcguard.required-check-gate.v1", owner=OWNER,
                decision="HOLD" if holds or failed else "PASS", required_checks=list(required), scope=SCOPE,
                engine=engine or {"name": "vllm", "version": "unknown"}, selected_arm=arm,
                total_planned_requests=total, selected_requests=len(rows),
                excluded_requests=total - len(rows) if type(total) is int else None,
                passed_requests=len(rows) - len(failed), hold_reasons=list(dict.fromkeys(holds)), requests=rows,
                runtime_qualified=False, combined_checks_supported=False)


# ------------------------------------------------------------------------------------------ recording evidence
def _cleanup_valid(v) -> bool:
    if (v.get("complete") is not True or v.get("errors") != [] or v.get("remaining_pids") != []
            or v.get("missing_terminal_evidence") != [] or v.get("roots_without_exact_exit_status") != []):
        return False
    members, terminal = v.get("process_membership"), v.get("terminal_handles")
    if type(members) is not list or not members or type(terminal) is not list:
        return False

    def ident(row):
        if type(row) is not dict or any(type(row.get(k)) is not int or row[k] <= 0 for k in ("pid", "start")):
            raise ValueError("invalid cleanup process identity")
        return row["pid"], row["start"]
    expected = [ident(r) for r in members]
    observed = [ident(r) for r in terminal if type(r) is dict and (
        (r.get("basis") == "same_pidfd_exit_readiness" and type(r.get("poll")) is dict
         and r["poll"].get("status") == "exit_observed")
        or (r.get("basis") == "exact_pidfd_wait" and type(r.get("returncode")) is int))]
    groups, sups = v.get("groups"), v.get("supervisor_receipts")
    if (type(groups) is not list or len(groups) != 2 or len(set(groups)) != 2
            or any(type(p) is not int or p <= 0 for p in groups) or type(sups) is not list or len(sups) != 2):
        return False
    by_term = {ident(r): r for r in terminal}
    reaped = v.get("reaped_leaders")
    if type(reaped) is not list or len(reaped) != len(groups):
        return False
    by_reap = {ident(r): r for r in reaped}
    roots = []
    for r in sups:
        if (r.get("complete") is not True or type(r.get("anchor_returncode")) is not int or r["anchor_returncode"] != 0
                or type(r.get("engine_returncode")) is not int or r["engine_returncode"] != 0):
            return False
        root = ident(r)
        ended, waited = by_term.get(root, {}), by_reap.get(root, {})
        if (ended.get("basis") != "exact_pidfd_wait" or type(ended.get("returncode")) is not int
                or ended["returncode"] != r["anchor_returncode"] or type(waited.get("returncode")) is not int
                or waited["returncode"] != r["anchor_returncode"]):
            return False
        roots.append(root)
    return (len(set(expected)) == len(expected) and len(set(observed)) == len(observed) and set(expected) == set(observed)
            and ev.same(sorted(v.get("observed_pids", [])), sorted(p for p, _ in expected))
            and sorted(p for p, _ in roots) == sorted(groups) and set(roots) <= set(expected))


def _startup_ok(v, plan, arm, role) -> bool:
    ctx = dict(run_id=plan["run_id"], packet_sha256=plan["packet_sha256"], arm_id=arm["arm_id"],
               engine_session_id=arm["engine_session_id"])
    rev = plan["source_revision"]
    want = dict(ctx, role=role, source_revision=rev, source_profile=profiles.client_source(rev), checksum_enabled=True,
                request_id_randomization_enabled=True, flashinfer_sampler_enabled=False, model_runner_v2=True,
                multiprocess_method="spawn", prefix_caching=plan.get("prefix_caching", False), chunked_prefill=True,
                async_scheduling=False, speculative_disabled=True, kv_dtype="auto", connector="NixlConnector",
                transfer_role="kv_producer" if role == "prefill" else "kv_consumer", block_size=16,
                max_model_len=2048, max_num_seqs=16, parallel=dict(tp=1, pp=1, dp=1, dcp=1, pcp=1),
                group_specs=[dict(type="FullAttentionSpec", block_size=16, sliding_window=None,
                                  attention_chunk_size=None, non_causal=False)])
    if "gpu_blocks_override" in plan:
        want["gpu_blocks"] = plan["gpu_blocks_override"]
    return (profiles.startup_supported(v, rev) and all(ev.same(v.get(k), x) for k, x in want.items())
            and type(v.get("process_id")) is int and v["process_id"] > 0
            and v.get("model") == plan["model"] == MODEL and v.get("model_revision") == MODEL_REVISION
            and v.get("dtype") in ("torch.bfloat16", "bfloat16"))


def _recording_issues(files, plan, captures) -> list[str]:
    """Bind the assembled inputs to the original startup receipts, close receipts and cleanup evidence."""
    issues, expected_native = [], set()
    for arm in plan["arms"]:
        aid = arm["arm_id"]
        startup = {}
        for role in ("prefill", "decode"):
            pre = aid + "/" + role + "/"
            paths = [n for n in files if n.startswith(pre + "startup-") and n.endswith(".json")]
            if len(paths) != 1:
                issues.append("startup_receipt_missing_or_ambiguous:" + pre)
                continue
            v = ev.object_at(files, paths[0])
            if v.get("checksum_enabled") is not True:
                issues.append("checksum_check_not_enabled:" + aid + ":" + role)
            if not _startup_ok(v, plan, arm, role) or paths[0] != pre + "startup-" + str(v.get("process_id")) + ".json":
                issues.append("unsupported_recorded_engine_config:" + pre)
            startup[role] = v
        cleanup = ev.object_at(files, aid + "/CLEANUP.json")
        if not _cleanup_valid(cleanup):
            issues.append("cleanup_evidence_incomplete:" + aid)
        members = {r["pid"] for r in cleanup.get("process_membership", []) if type(r) is dict and type(r.get("pid")) is int}
        for role, v in startup.items():
            if v.get("process_id") not in members:
                issues.append("startup_process_membership_unverified:" + aid + ":" + role)
        if not arm["observer_enabled"]:
            continue
        sel = [c for c in captures["captures"] if c.get("arm_id") == aid]
        if len(sel) != 1:
            issues.append("capture_missing_or_ambiguous:" + aid)
            continue
        cap = sel[0]
        envs = [("decode", cap)]
        if plan.get("prefix_caching") is True:
            envs.append(("prefill", cap.get("prefill_capture", {})))
        for role, env in envs:
            env = env if type(env) is dict else {}
            asm = env.get("startup", {})
            asm = asm if type(asm) is dict else {}
            if not ev.same({k: x for k, x in asm.items() if k != "native_transport"}, startup.get(role)):
                issues.append("startup_assembly_disagrees:" + aid + ":" + role)
            if env.get("capture_complete") is not True or env.get("capture_errors") != []:
                issues.append("native_capture_incomplete:" + aid + ":" + role)
            pre = aid + "/" + role + "/"
            kinds = [("bindings", "binding_snapshots")]
            if role == "decode":
                kinds.insert(0, ("checksum", "checksum_snapshots"))
            if plan.get("prefix_caching") is True:
                kinds.append(("cache", "cache_snapshots"))
            for kind, key in kinds:
                paths = sorted(n for n in files if n.startswith(pre + kind + "-") and n.endswith(".json")
                               and "-disabled-" not in n)
                originals = []
                for name in paths:
                    expected_native.add(name)
                    v = ev.object_at(files, name)
                    ctx = v.get("context", {})
                    pid = ctx.get("process_id") if type(ctx) is dict else None
                    want_ctx = {k: plan[k] if k in ("run_id", "packet_sha256") else arm[k] for k in CONTEXT}
                    want_ctx["process_id"] = pid
                    if (type(pid) is not int or pid <= 0 or name != pre + kind + "-" + str(pid) + ".json"
                            or not ev.same(ctx, want_ctx) or v.get("role") != role
                            or v.get("schema") != "sdcguard.owner-checksum-close.v1"
                            or v.get("original_shutdown_completed") is not True
                            or v.get("original_shutdown_error") is not None or v.get("recorder_errors") != []):
                        issues.append("native_close_receipt_unverified:" + name)
                    snap = v.get("snapshot")
                    if type(snap) is not dict or snap.get("qualification") != "source_bound_candidate":
                        issues.append("non_runtime_native_evidence:" + name)
                    sctx = ((snap.get("capture_context") if kind == "checksum" else
                             {k: snap.get(k) for k in (*CONTEXT, "process_id")}) if type(snap) is dict else None)
                    if not ev.same(sctx, want_ctx):
                        issues.append("native_snapshot_context_disagrees:" + name)
                    if kind in ("checksum", "cache") and pid != startup.get(role, {}).get("process_id"):
                        issues.append("native_scheduler_process_disagrees:" + name)
                    if kind == "cache" and (type(snap) is not dict or snap.get("role") != role):
                        issues.append("native_cache_role_disagrees:" + name)
                    if pid not in members:
                        issues.append("native_recorder_process_membership_unverified:" + name)
                    originals.append(snap)
                if not originals or not ev.same(originals, env.get(key)):
                    issues.append("native_snapshot_assembly_disagrees:" + aid + ":" + role + ":" + kind)
    for name in files:
        base = name.rsplit("/", 1)[-1]
        if base.startswith("errors-") and name.endswith(".json"):
            issues.append("native_recorder_error:" + name)
        if (base.startswith(("checksum-", "bindings-", "cache-")) and name.endswith(".json")
                and "-disabled-" not in base and name not in expected_native):
            issues.append("unexpected_native_receipt:" + name)
    return issues


def _journal_issues(files) -> list[str]:
    """Client stage journal: every planned stage started then finished exactly once, with the planned request,
    and each prefill finished before its decode started."""
    inv = ev.object_at(files, "client/CLIENT_INVENTORY.json")
    want = {(r["arm_id"], r["slot"], role): r[role] for r in inv["requests"] for role in ("prefill", "decode")}
    started, finished = {}, {}
    lines = files.get("client/CLIENT_RECEIPTS.jsonl", b"").splitlines()
    if len(lines) != 2 * len(want):
        return ["client_journal_stage_count_disagrees"]
    for seq, raw in enumerate(lines, 1):
        v = ev.parse_json(raw)
        if (type(v) is not dict or type(v.get("sequence")) is not int or v["sequence"] != seq
                or type(v.get("slot")) is not int or type(v.get("arm_id")) is not str
                or v.get("role") not in ("prefill", "decode")):
            return ["client_journal_sequence_unverified"]
        k = v["arm_id"], v["slot"], v["role"]
        rc = v.get("receipt")
        if k not in want or type(rc) is not dict:
            return ["client_journal_unplanned_stage"]
        if v.get("kind") == "stage_started":
            if (k in started or rc.get("completed") is not False or rc.get("http_status") is not None
                    or rc.get("error") is not None or rc.get("response_body") is not None
                    or any(not ev.same(rc.get(x), want[k].get(x)) for x in ("method", "path", "request_body",
                                                                          "request_headers"))):
                return ["client_journal_started_stage_disagrees"]
            started[k] = seq
        elif v.get("kind") == "stage_finished":
            if k not in started or k in finished or not ev.same(rc, want[k]):
                return ["client_journal_finished_stage_disagrees"]
            finished[k] = seq
        else:
            return ["client_journal_kind_unverified"]
    if set(started) != set(want) or set(finished) != set(want):
        return ["client_journal_incomplete"]
    if any(finished[a, s, "prefill"] >= started[a, s, "decode"] for a, s, role in want if role == "prefill"):
        return ["client_journal_handoff_order_unverified"]
    return []


def _installed_witness(v) -> dict:
    return dict(schema=INSTALLED_WITNESS, packet_sha256=v["packet_sha256"], run_id=v["run_id"],
                plan_sha256=v["plan_sha256"], installed_identity_sha256=ev.digest(ev.json_bytes(v["installed_engine"])),
                product_identity_sha256=ev.digest(ev.json_bytes(v["product"])),
                preflight_sha256=ev.digest(ev.json_bytes({k: x for k, x in v.items()
                                                          if k not in ("build_witness", "build_witness_sha256")})),
                runtime_qualified=False,
                scope="observed installed bytes and CPU prerequisites; no execution attestation")


def _installed_preflight_ok(v, plan, plan_raw) -> bool:
    """Internal consistency of an installed-runtime preflight: identity, pinned engine version and a build
    witness that hashes the preflight it is part of."""
    try:
        rev = plan["source_revision"]
        sel = profiles.get(rev)
        if (type(v) is not dict or v.get("schema") != INSTALLED_SCHEMA or v.get("status") != "PASS"
                or v.get("failure") is not None or v.get("cpu_only") is not True or v.get("gpu_submitted") is not False
                or v.get("runtime_qualified") is not False or v.get("run_id") != plan["run_id"]
                or v.get("packet_sha256") != plan["packet_sha256"] or v.get("plan_sha256") != ev.digest(plan_raw)
                or v.get("source_revision") != rev):
            return False
        product, engine = v["product"], v["installed_engine"]
        if (product.get("sha256") != ev.digest(ev.json_bytes(product["files"])) or product["sha256"] != plan["packet_sha256"]
                or engine.get("schema") != "sdcguard.owner-checksum-installed.v1" or engine.get("source_revision") != rev
                or engine.get("runtime_qualified") is not False or engine["versions"]["vllm"] != sel["version"]):
            return False
        source = v["pinned_source_guard"]
        if source.get("head") != rev or source.get("tracked_status") != "":
            return False
        mc = v["model_cache"]
        if mc.get("model") != MODEL or mc.get("revision") != MODEL_REVISION or type(mc.get("snapshot")) is not str \
                or not mc["snapshot"].startswith("/") or Path(mc["snapshot"]).name != MODEL_REVISION:
            return False
        if not ev.same(v["python_runtime"]["identity"], engine["python_identity"]):
            return False
        w = _installed_witness(v)
        return ev.json_bytes(v["build_witness"]) == ev.json_bytes(w) and v.get("build_witness_sha256") == ev.digest(
            ev.json_bytes(w))
    except (ValueError, KeyError, TypeError, AttributeError):
        return False


def checksum_gate(result_raw: bytes, archive_raw: bytes, preflight_raw, required, arm=None) -> dict:
    result, files = ev.parse_json(result_raw), ev.read_archive(archive_raw)
    consumed = {n: r for n, r in files.items() if n in (
        "client/REQUEST_PLAN.json", "client/CLIENT_INVENTORY.json", "client/CLIENT_RECEIPTS.jsonl", "CAPTURES.json",
        "FINISHED.json", "BUILD_WITNESS.json") or n.endswith("/CLEANUP.json")
        or n.rsplit("/", 1)[-1].startswith(("startup-", "checksum-", "bindings-", "cache-"))}
    if preflight_raw is not None:
        consumed["CPU_PREFLIGHT.json"] = preflight_raw
    consumed["RESULT.json"] = result_raw
    ev.count_nodes(consumed, max_nodes=ev.MAX_TOTAL_JSON_NODES)
    plan = ev.object_at(files, "client/REQUEST_PLAN.json")
    captures = ev.object_at(files, "CAPTURES.json")
    report = cl.evaluate(files["client/REQUEST_PLAN.json"], files["client/CLIENT_INVENTORY.json"], files["CAPTURES.json"])
    issues = [x for x in report["hold_reasons"] if x not in cl.PROFILE_LIMITS and x != COVERAGE_HOLD]
    finished = ev.object_at(files, "FINISHED.json")
    if (not ev.same(result.get("report"), finished) or result.get("archive_sha256") != ev.digest(archive_raw)
            or any(not ev.same(result.get(k), plan[k]) for k in ("run_id", "packet_sha256"))
            or any(not ev.same(finished.get(k), plan[k]) for k in ("run_id", "packet_sha256"))):
        issues.append("owner_evidence_identity_disagrees")
    if (finished.get("complete") is not True or finished.get("failure") is not None
            or finished.get("stage") != "complete" or finished.get("cleanup_complete") is not True
            or finished.get("client_inventory_complete") is not True):
        issues.append("owner_run_completion_unverified")
    version, recorded_rev = "unknown", "unknown"
    if preflight_raw is None:
        issues.append("recorded_engine_build_missing")
    else:
        pre = ev.parse_json(preflight_raw)
        inst = pre.get("installed_engine", {})
        version = inst.get("versions", {}).get("vllm", "unknown")
        recorded_rev = inst.get("source_revision", "unknown")
        witness = ev.object_at(files, "BUILD_WITNESS.json")
        payload = witness.get("witness", {})
        rev = plan["source_revision"]
        if version != profiles.get(rev)["version"] or inst.get("source_revision") != rev or pre.get("source_revision") != rev:
            issues.append("unsupported_recorded_engine_version")
        if pre.get("schema") == INSTALLED_SCHEMA:
            if (not _installed_preflight_ok(pre, plan, files["client/REQUEST_PLAN.json"])
                    or payload.get("schema") != INSTALLED_WITNESS or not ev.same(payload, pre.get("build_witness"))
                    or witness.get("sha256") != pre.get("build_witness_sha256")
                    or result.get("build_witness_sha256") != witness.get("sha256")):
                issues.append("installed_runtime_preflight_unverified")
            snap = pre.get("model_cache", {}).get("snapshot")
            for parm in plan["arms"]:
                for role in ("prefill", "decode"):
                    p = parm["arm_id"] + "/" + role + "/startup-"
                    starts = [ev.object_at(files, n) for n in files if n.startswith(p) and n.endswith(".json")]
                    if len(starts) != 1 or type(snap) is not str or any(
                            starts[0].get(k) != snap for k in ("actual_model", "actual_tokenizer", "snapshot")):
                        issues.append("installed_model_startup_binding_unverified:" + parm["arm_id"] + ":" + role)
        elif rev != profiles.BASELINE:
            issues.append("candidate_requires_installed_runtime_preflight")
        elif (witness.get("sha256") != ev.digest(ev.json_bytes(payload))
              or result.get("build_witness_sha256") != witness.get("sha256")
              or payload.get("schema") != "sdcguard.owner-checksum-build-witness.v1"
              or payload.get("installed_identity_sha256") != ev.digest(ev.json_bytes(inst))
              or payload.get("packet_sha256") != plan["packet_sha256"] or pre.get("packet_sha256") != plan["packet_sha256"]
              or pre.get("run_id") != plan["run_id"] or pre.get("status") != "PASS"
              or pre.get("schema") != "sdcguard.owner-checksum-cpu-preflight.v1"
              or inst.get("schema") != "sdcguard.owner-checksum-installed.v1" or pre.get("failure") is not None
              or pre.get("plan_sha256") != ev.digest(files["client/REQUEST_PLAN.json"])
              or not ev.same(pre.get("build_witness"), payload)
              or pre.get("build_witness_sha256") != witness.get("sha256")
              or any(pre.get(k) != payload.get(k) for k in ("build_result_sha256", "build_archive_sha256"))
              or payload.get("pinned_source_guard_sha256") != ev.digest(ev.json_bytes(pre.get("pinned_source_guard")))
              or payload.get("python_identity_sha256") != ev.digest(ev.json_bytes(
                  pre.get("python_runtime", {}).get("identity")))):
            issues.append("recorded_engine_build_unverified")
    issues.extend(_recording_issues(files, plan, captures))
    issues.extend(_journal_issues(files))
    domains = {a["arm_id"]: "source_bound_candidate" if a["observer_enabled"] else "observer_disabled"
               for a in plan["arms"]}
    if any(c["qualification"] != domains.get(c["arm_id"]) for c in report["captures"]):
        issues.append("runtime_capture_source_unverified")
    rows = []
    for row in report["requests"]:
        if arm is not None and row["arm_id"] != arm:
            continue
        calls = row["checksum_calls"]
        proof = calls[0]["conditional_scope"] if len(calls) == 1 else {}
        check = dict(native_result=row["native_result"], expected_units=proof.get("expected_units"),
                     compared_units=proof.get("compared_units"),
                     completed=len(calls) == 1 and row["check_status"] == "passed",
                     evidence_complete=row["coverage"] == "complete" and not row["reasons"],
                     applicable=row["observer_enabled"],
                     reason=row["reasons"][0] if row["reasons"] else "complete_recorded_comparison")
        rows.append(dict(client_request_id=row["client_request_id"], arm_id=row["arm_id"], slot=row["slot"],
                         checks={"checksum": check}, token_coverage=row["token_coverage"], reasons=list(row["reasons"])))
    if arm is not None and arm not in {a["arm_id"] for a in plan["arms"]}:
        issues.append("selected_arm_not_in_plan")
    ans = decide(rows, required, issues, total=len(report["requests"]),
                 engine=dict(name="vllm", version=version, source_revision=recorded_rev,
                             supported_source_revision=plan["source_revision"]), arm=arm)
    if COVERAGE_HOLD in report["hold_reasons"]:
        ans["decision"] = "HOLD"
        ans["hold_reasons"].insert(0, COVERAGE_HOLD)
    return ans


def inspect(path, required, arm=None) -> dict:
    path = Path(path)
    from . import own
    if path.is_dir() and own.is_own_recording(path):
        return own.inspect(path)
    if path.is_file():
        ev.parse_json(ev.read_file(path.parent, path.name))
        return decide([], required, ["legacy_summary_has_no_complete_per_request_check_evidence"], arm=arm)
    result = ev.read_file(path, "RESULT.json")
    archive = ev.read_file(path, "ordinary-evidence.zip")
    files = ev.read_archive(archive)
    if "client/REQUEST_PLAN.json" in files:
        pre = ev.read_file(path, "CPU_PREFLIGHT.json") if (path / "CPU_PREFLIGHT.json").exists() else None
        ans = checksum_gate(result, archive, pre, required, arm)
        if pre is not None and pre != ev.read_file(path, "CPU_PREFLIGHT.json"):
            raise ev.EvidenceError("engine build evidence changed during inspection")
    else:
        ans = decide([], required, ["unsupported_recorded_engine_profile"], arm=arm)
    if result != ev.read_file(path, "RESULT.json") or archive != ev.read_file(path, "ordinary-evidence.zip"):
        raise ev.EvidenceError("owner inputs changed during inspection")
    return ans


def render(ans: dict) -> str:
    lines = [ans["decision"] + " | required: " + ", ".join(ans["required_checks"]), ans["scope"],
             f"{ans['passed_requests']} / {ans['selected_requests']} selected requests passed",
             f"Total planned: {ans['total_planned_requests']}; explicitly excluded: {ans['excluded_requests']}"]
    lines.extend("HOLD: " + r for r in ans["hold_reasons"])
    for row in ans["requests"]:
        lines.append(f"{row['client_request_id']} | {row['decision']} | "
                     + ("; ".join(row["reasons"]) or "required check passed with complete recorded coverage"))
        t = row.get("token_coverage")
        if type(t) is dict:
            def n(k):
                v = t.get(k)
                return str(v) if type(v) is int else "unknown"
            lines.append(f"  Prompt tokens: {n('prompt_tokens')}; transferred tokens checked: "
                         f"{n('transferred_tokens_checked')}; decode cache reused unchecked: "
                         f"{n('decode_cached_tokens_unchecked')}; prefill cache reused: {n('prefill_cached_tokens')}")
    return "\n".join(lines) + "\n"


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="sdcguard gate", description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("input", help="saved owner-result directory or historical RESULT.json")
    ap.add_argument("--require", choices=CHECKS, action="append", required=True)
    ap.add_argument("--arm", help="explicit checksum workload arm; default includes all planned requests")
    ap.add_argument("--json", action="store_true")
    a = ap.parse_args(argv)
    try:
        ans = inspect(a.input, a.require, a.arm)
    except (ValueError, OSError, KeyError, TypeError, AttributeError) as e:
        ans = decide([], list(dict.fromkeys(a.require)), ["evidence_unverifiable:" + str(e)], arm=a.arm)
    sys.stdout.write(ev.json_bytes(ans).decode() if a.json else render(ans))
    return 0 if ans["decision"] == "PASS" else 2
