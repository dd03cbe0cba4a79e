"""`sdcguard gate DIR --require checksum`: offline per-request coverage gate over a recorded prefill/decode run.

PASS applies to the selected recorded requests and check only: a request passes when the native KV checksum
compared its whole prompt and every piece of evidence that binds the comparison to that request is intact.
Anything unverifiable holds. Exit 0 on PASS, 2 on HOLD. Nothing is executed and no device is used.

Inputs (a recorded owner-result directory): RESULT.json, ordinary-evidence.zip (request plan, client inventory and
journal, engine captures, close receipts, cleanup evidence) and CPU_PREFLIGHT.json (engine build identity).

Verdict rules, reason strings and the text rendering keep the reference's contract (src/sdcguard/required_gate.py:
68-490, native_checks.py:54-93) so that saved recordings give the same verdicts. Here the recording is audited by
small readers, each owning one kind of evidence and emitting its findings in a fixed order: `_run_issues` (run
identity and completion), `_build_issues` (engine build), `_ReceiptAudit` (startup receipts, cleanup via `_Cleanup`,
native close receipts), `_Journal` (client stage order); the per-check policy is `assess_check` with the reasons of
a check that did not pass as an ordered table (`_NOT_PASSED`).
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


def _coverage(exp, cmp_, evidence_complete, applicable) -> str:
    if exp is None or cmp_ is None or not evidence_complete:
        return "unknown"
    if not exp or not cmp_ or applicable is False:
        return "not_covered"
    return "partial" if set(exp) - set(cmp_) else "complete"


# why an applicable check did not pass, first match wins: (the check's state -> bool, reason)
_NOT_PASSED = (
    (lambda c: not c["evidence_complete"], "recording_incomplete"),
    (lambda c: c["expected_units"] is None, "expected_scope_unknown"),
    (lambda c: not c["expected_units"], "no_eligible_comparison_units"),
    (lambda c: c["coverage"] == "partial", "comparison_scope_partial"),
    (lambda c: not c["compared_units"], "no_recorded_comparison"),
    (lambda c: not c["completed"], "comparison_not_completed"),
    (lambda c: True, "no_recorded_passing_result"),
)


def assess_check(check_id, *, native_result, expected_units, compared_units, completed, evidence_complete,
                 applicable=True, reason=None) -> dict:
    """Status of one check from normalised facts: passed only with a passing native result, completed call,
    complete evidence and complete coverage of the eligible units."""
    if check_id not in CHECKS or native_result not in NATIVE_RESULTS:
        raise ValueError("unsupported check or native result")
    typed = (type(completed) is bool and type(evidence_complete) is bool
             and (applicable is None or type(applicable) is bool)
             and (reason is None or (type(reason) is str and reason and len(reason) <= 1024)))
    if not typed:
        raise ValueError("explicit boolean completion and bounded reason are required")
    exp, cmp_ = _units(expected_units, "expected_units"), _units(compared_units, "compared_units")
    if exp is not None and cmp_ is not None and not set(cmp_) <= set(exp):
        raise ValueError("compared units include units outside the eligible scope")
    c = {"check": check_id, "native_result": native_result, "coverage": _coverage(exp, cmp_, evidence_complete,
                                                                                 applicable),
         "expected_units": exp, "compared_units": cmp_,
         "missing_units": sorted(set(exp) - set(cmp_ or ())) if exp is not None else None,
         "completed": completed, "evidence_complete": evidence_complete, "applicable": applicable}
    if applicable is not True:
        status, why = "unverified", reason or ("not_applicable" if applicable is False else "applicability_unknown")
    elif native_result == "mismatch" and evidence_complete and completed and cmp_:
        status, why = "mismatch", reason or "recorded_native_mismatch"
    elif native_result == "passed" and completed and evidence_complete and c["coverage"] == "complete":
        status, why = "passed", reason or "complete_recorded_comparison"
    else:
        status, why = "unverified", reason or next(r for test, r in _NOT_PASSED if test(c))
    c.update(check_status=status, coverage_complete=c["coverage"] == "complete", reason=why)
    return c


def _request_row(rq: dict, required, holds: list) -> dict:
    """One request under the required checks: its own reasons, one per required check that did not pass, and
    the gate-wide holds."""
    reasons = list(rq.get("reasons", []))
    for name in required:
        item = rq.get("checks", {}).get(name)
        if type(item) is not dict:
            reasons.append(name + ":not_recorded")
        elif item.get("check", name) != name:
            reasons.append(name + ":different_check_recorded")
        else:
            a = assess_check(name, native_result=item.get("native_result", "unverified"),
                             expected_units=item.get("expected_units"), compared_units=item.get("compared_units"),
                             completed=item.get("completed") is True,
                             evidence_complete=item.get("evidence_complete") is True,
                             applicable=item.get("applicable"), reason=item.get("reason"))
            if a["check_status"] != "passed":
                reasons.append(name + ":" + a["reason"])
    every = list(dict.fromkeys(reasons + holds))
    return dict(rq, decision="HOLD" if every else "PASS", reasons=every)


def decide(requests, required, issues=(), *, total=None, engine=None, arm=None) -> dict:
    """Apply the required-check policy to per-request facts; supplied statuses are never trusted."""
    if not required or any(c not in CHECKS for c in required) or len(set(required)) != len(required):
        raise ev.EvidenceError("require lease, checksum, or both once each")
    holds = list(issues)
    holds += [r for r, bad in (("combined_lease_checksum_not_supported", len(required) != 1),
                               ("no_verified_request_denominator", not requests)) if bad]
    rows = [_request_row(rq, required, holds) for rq in requests]
    held = sum(r["decision"] == "HOLD" for r in rows)
    return dict(schema="sdcguard.required-check-gate.v1", owner=OWNER,
                decision="HOLD" if holds or held else "PASS", required_checks=list(required), scope=SCOPE,
                engine=engine or {"name": "vllm", "version": "unknown"}, selected_arm=arm,
                total_planned_requests=total, selected_requests=len(rows),
                excluded_requests=total - len(rows) if type(total) is int else None,
                passed_requests=len(rows) - held, hold_reasons=list(dict.fromkeys(holds)), requests=rows,
                runtime_qualified=False, combined_checks_supported=False)


# ------------------------------------------------------------------------------------------ recording evidence
def _pid_start(row) -> tuple:
    """(pid, start time) of a recorded process; a malformed identity makes the cleanup evidence unreadable."""
    if type(row) is not dict or any(type(row.get(k)) is not int or row[k] <= 0 for k in ("pid", "start")):
        raise ValueError("invalid cleanup process identity")
    return row["pid"], row["start"]


def _exit_seen(row) -> bool:
    """A terminal handle that shows the process exit (its pidfd became readable, or an exact wait returned)."""
    if type(row) is not dict:
        return False
    if row.get("basis") == "same_pidfd_exit_readiness":
        return type(row.get("poll")) is dict and row["poll"].get("status") == "exit_observed"
    return row.get("basis") == "exact_pidfd_wait" and type(row.get("returncode")) is int


class _Cleanup:
    """The arm's process cleanup evidence: every member process of both engine groups exited and was seen to
    exit, and each group's supervisor anchor ended with the exact status its supervisor reported."""

    def __init__(self, v: dict):
        self.v = v

    def valid(self) -> bool:
        v = self.v
        if not (v.get("complete") is True and all(v.get(k) == [] for k in (
                "errors", "remaining_pids", "missing_terminal_evidence", "roots_without_exact_exit_status"))):
            return False
        members, terminal = v.get("process_membership"), v.get("terminal_handles")
        if type(members) is not list or not members or type(terminal) is not list:
            return False
        expected = [_pid_start(r) for r in members]
        observed = [_pid_start(r) for r in terminal if _exit_seen(r)]
        groups, sups = v.get("groups"), v.get("supervisor_receipts")
        if not (type(groups) is list and len(groups) == 2 and len(set(groups)) == 2
                and all(type(g) is int and g > 0 for g in groups) and type(sups) is list and len(sups) == 2):
            return False
        ended = {_pid_start(r): r for r in terminal}
        reaped = v.get("reaped_leaders")
        if type(reaped) is not list or len(reaped) != len(groups):
            return False
        waited = {_pid_start(r): r for r in reaped}
        roots = []
        for r in sups:
            if not self._anchor_ok(r, ended, waited):
                return False
            roots.append(_pid_start(r))
        exp_set = set(expected)
        return (len(exp_set) == len(expected) and len(set(observed)) == len(observed) and exp_set == set(observed)
                and ev.same(sorted(v.get("observed_pids", [])), sorted(p for p, _ in expected))
                and sorted(p for p, _ in roots) == sorted(groups) and set(roots) <= exp_set)

    @staticmethod
    def _anchor_ok(r, ended: dict, waited: dict) -> bool:
        rc = r.get("anchor_returncode")
        if not (r.get("complete") is True and type(rc) is int and rc == 0
                and type(r.get("engine_returncode")) is int and r["engine_returncode"] == 0):
            return False
        root = _pid_start(r)
        e, w = ended.get(root, {}), waited.get(root, {})
        return (e.get("basis") == "exact_pidfd_wait" and type(e.get("returncode")) is int and e["returncode"] == rc
                and type(w.get("returncode")) is int and w["returncode"] == rc)


def _cleanup_valid(v) -> bool:
    return _Cleanup(v).valid()


def _expected_startup(plan, arm, role) -> dict:
    """The startup receipt a supported engine of this arm and role writes (its configuration as pinned)."""
    rev = plan["source_revision"]
    want = dict(run_id=plan["run_id"], packet_sha256=plan["packet_sha256"], arm_id=arm["arm_id"],
                engine_session_id=arm["engine_session_id"], role=role, source_revision=rev,
                source_profile=profiles.client_source(rev), checksum_enabled=True,
                request_id_randomization_enabled=True, flashinfer_sampler_enabled=False, model_runner_v2=True,
                multiprocess_method="spawn", prefix_caching=plan.get("prefix_caching", False), chunked_prefill=True,
                async_scheduling=False, speculative_disabled=True, kv_dtype="auto", connector="NixlConnector",
                transfer_role="kv_producer" if role == "prefill" else "kv_consumer", block_size=16,
                max_model_len=2048, max_num_seqs=16, parallel=dict(tp=1, pp=1, dp=1, dcp=1, pcp=1),
                group_specs=[dict(type="FullAttentionSpec", block_size=16, sliding_window=None,
                                  attention_chunk_size=None, non_causal=False)])
    if "gpu_blocks_override" in plan:
        want["gpu_blocks"] = plan["gpu_blocks_override"]
    return want


def _startup_ok(v, plan, arm, role) -> bool:
    want = _expected_startup(plan, arm, role)
    return (profiles.startup_supported(v, plan["source_revision"]) and all(ev.same(v.get(k), x) for k, x in want.items())
            and type(v.get("process_id")) is int and v["process_id"] > 0
            and v.get("model") == plan["model"] == MODEL and v.get("model_revision") == MODEL_REVISION
            and v.get("dtype") in ("torch.bfloat16", "bfloat16"))


class _ReceiptAudit:
    """Binds the assembled inputs of a recording to its original receipts: each engine's startup receipt, the
    arm's cleanup evidence, and every native recorder's close receipt (context, closure, snapshot). Findings come
    out in a fixed order: per arm (startups, cleanup, memberships, then the observed arm's capture and receipts),
    then files that no audit expected."""

    KINDS = {"checksum": "checksum_snapshots", "bindings": "binding_snapshots", "cache": "cache_snapshots"}

    def __init__(self, files: dict, plan: dict, captures: dict):
        self.files, self.plan, self.captures = files, plan, captures
        self.expected_native: set = set()
        self.out: list[str] = []

    def run(self) -> list[str]:
        for arm in self.plan["arms"]:
            self._arm(arm)
        self._stray_files()
        return self.out

    def _named(self, prefix: str) -> list[str]:
        return [n for n in self.files if n.startswith(prefix) and n.endswith(".json")]

    def _arm(self, arm) -> None:
        aid = arm["arm_id"]
        startup = self._startups(arm)
        cleanup = ev.object_at(self.files, aid + "/CLEANUP.json")
        if not _cleanup_valid(cleanup):
            self.out.append("cleanup_evidence_incomplete:" + aid)
        members = {r["pid"] for r in cleanup.get("process_membership", [])
                   if type(r) is dict and type(r.get("pid")) is int}
        self.out += ["startup_process_membership_unverified:" + aid + ":" + role
                     for role, v in startup.items() if v.get("process_id") not in members]
        if not arm["observer_enabled"]:
            return
        mine = [c for c in self.captures["captures"] if c.get("arm_id") == aid]
        if len(mine) != 1:
            self.out.append("capture_missing_or_ambiguous:" + aid)
            return
        cap = mine[0]
        envs = [("decode", cap)]
        if self.plan.get("prefix_caching") is True:
            envs.append(("prefill", cap.get("prefill_capture", {})))
        for role, env in envs:
            self._engine_capture(arm, role, env if type(env) is dict else {}, startup, members)

    def _startups(self, arm) -> dict:
        aid, found = arm["arm_id"], {}
        for role in ("prefill", "decode"):
            pre = aid + "/" + role + "/"
            paths = self._named(pre + "startup-")
            if len(paths) != 1:
                self.out.append("startup_receipt_missing_or_ambiguous:" + pre)
                continue
            v = ev.object_at(self.files, paths[0])
            if v.get("checksum_enabled") is not True:
                self.out.append("checksum_check_not_enabled:" + aid + ":" + role)
            if not _startup_ok(v, self.plan, arm, role) or paths[0] != pre + "startup-" + str(v.get("process_id")) + ".json":
                self.out.append("unsupported_recorded_engine_config:" + pre)
            found[role] = v
        return found

    def _engine_capture(self, arm, role, env: dict, startup: dict, members: set) -> None:
        aid = arm["arm_id"]
        asm = env.get("startup", {})
        asm = asm if type(asm) is dict else {}
        if not ev.same({k: x for k, x in asm.items() if k != "native_transport"}, startup.get(role)):
            self.out.append("startup_assembly_disagrees:" + aid + ":" + role)
        if env.get("capture_complete") is not True or env.get("capture_errors") != []:
            self.out.append("native_capture_incomplete:" + aid + ":" + role)
        kinds = (["checksum"] if role == "decode" else []) + ["bindings"]
        if self.plan.get("prefix_caching") is True:
            kinds.append("cache")
        for kind in kinds:
            self._receipts(arm, role, kind, env, startup, members)

    def _context(self, arm, pid) -> dict:
        ctx = {k: self.plan[k] if k in ("run_id", "packet_sha256") else arm[k] for k in CONTEXT}
        ctx["process_id"] = pid
        return ctx

    def _receipts(self, arm, role, kind, env, startup, members) -> None:
        aid, pre = arm["arm_id"], arm["arm_id"] + "/" + role + "/"
        paths = sorted(n for n in self._named(pre + kind + "-") if "-disabled-" not in n)
        originals = []
        for name in paths:
            self.expected_native.add(name)
            v = ev.object_at(self.files, name)
            ctx = v.get("context", {})
            pid = ctx.get("process_id") if type(ctx) is dict else None
            want = self._context(arm, pid)
            closed = (type(pid) is int and pid > 0 and name == pre + kind + "-" + str(pid) + ".json"
                      and ev.same(ctx, want) and v.get("role") == role
                      and v.get("schema") == "sdcguard.owner-checksum-close.v1"
                      and v.get("original_shutdown_completed") is True and v.get("original_shutdown_error") is None
                      and v.get("recorder_errors") == [])
            snap = v.get("snapshot")
            snap_ok = type(snap) is dict
            seen_ctx = ((snap.get("capture_context") if kind == "checksum" else
                         {k: snap.get(k) for k in (*CONTEXT, "process_id")}) if snap_ok else None)
            for reason, bad in (
                    ("native_close_receipt_unverified:", not closed),
                    ("non_runtime_native_evidence:", not snap_ok or snap.get("qualification") != "source_bound_candidate"),
                    ("native_snapshot_context_disagrees:", not ev.same(seen_ctx, want)),
                    ("native_scheduler_process_disagrees:",
                     kind in ("checksum", "cache") and pid != startup.get(role, {}).get("process_id")),
                    ("native_cache_role_disagrees:", kind == "cache" and (not snap_ok or snap.get("role") != role)),
                    ("native_recorder_process_membership_unverified:", pid not in members)):
                if bad:
                    self.out.append(reason + name)
            originals.append(snap)
        if not originals or not ev.same(originals, env.get(self.KINDS[kind])):
            self.out.append("native_snapshot_assembly_disagrees:" + aid + ":" + role + ":" + kind)

    def _stray_files(self) -> None:
        for name in self.files:
            base = name.rsplit("/", 1)[-1]
            if not name.endswith(".json"):
                continue
            if base.startswith("errors-"):
                self.out.append("native_recorder_error:" + name)
            if (base.startswith(("checksum-", "bindings-", "cache-")) and "-disabled-" not in base
                    and name not in self.expected_native):
                self.out.append("unexpected_native_receipt:" + name)


def _recording_issues(files, plan, captures) -> list[str]:
    """Bind the assembled inputs to the original startup receipts, close receipts and cleanup evidence."""
    return _ReceiptAudit(files, plan, captures).run()


class _Journal:
    """The client's stage journal: every planned stage started then finished exactly once, as planned, and each
    request's prefill finished before its decode started. The first broken rule is the only finding."""

    def __init__(self, files: dict):
        inv = ev.object_at(files, "client/CLIENT_INVENTORY.json")
        self.want = {(r["arm_id"], r["slot"], role): r[role] for r in inv["requests"] for role in ("prefill", "decode")}
        self.lines = files.get("client/CLIENT_RECEIPTS.jsonl", b"").splitlines()
        self.started: dict = {}
        self.finished: dict = {}

    def issue(self):
        if len(self.lines) != 2 * len(self.want):
            return "client_journal_stage_count_disagrees"
        for seq, raw in enumerate(self.lines, 1):
            bad = self._entry(seq, ev.parse_json(raw))
            if bad:
                return bad
        if set(self.started) != set(self.want) or set(self.finished) != set(self.want):
            return "client_journal_incomplete"
        if any(self.finished[a, s, "prefill"] >= self.started[a, s, "decode"] for a, s, role in self.want
               if role == "prefill"):
            return "client_journal_handoff_order_unverified"
        return None

    def _entry(self, seq: int, v):
        if not (type(v) is dict and type(v.get("sequence")) is int and v["sequence"] == seq
                and type(v.get("slot")) is int and type(v.get("arm_id")) is str and v.get("role") in ("prefill", "decode")):
            return "client_journal_sequence_unverified"
        k, rc = (v["arm_id"], v["slot"], v["role"]), v.get("receipt")
        if k not in self.want or type(rc) is not dict:
            return "client_journal_unplanned_stage"
        kind = v.get("kind")
        if kind == "stage_started":
            fresh = (k not in self.started and rc.get("completed") is False
                     and all(rc.get(x) is None for x in ("http_status", "error", "response_body"))
                     and all(ev.same(rc.get(x), self.want[k].get(x))
                             for x in ("method", "path", "request_body", "request_headers")))
            if not fresh:
                return "client_journal_started_stage_disagrees"
            self.started[k] = seq
        elif kind == "stage_finished":
            if k not in self.started or k in self.finished or not ev.same(rc, self.want[k]):
                return "client_journal_finished_stage_disagrees"
            self.finished[k] = seq
        else:
            return "client_journal_kind_unverified"
        return None


def _journal_issues(files) -> list[str]:
    """Client stage journal: every planned stage started then finished exactly once, with the planned request,
    and each prefill finished before its decode started."""
    bad = _Journal(files).issue()
    return [bad] if bad else []


def _canon_digest(v) -> str:
    return ev.digest(ev.json_bytes(v))


def _installed_witness(v) -> dict:
    return dict(schema=INSTALLED_WITNESS, packet_sha256=v["packet_sha256"], run_id=v["run_id"],
                plan_sha256=v["plan_sha256"], installed_identity_sha256=_canon_digest(v["installed_engine"]),
                product_identity_sha256=_canon_digest(v["product"]),
                preflight_sha256=_canon_digest({k: x for k, x in v.items()
                                                if k not in ("build_witness", "build_witness_sha256")}),
                runtime_qualified=False,
                scope="observed installed bytes and CPU prerequisites; no execution attestation")


def _installed_preflight_ok(v, plan, plan_raw) -> bool:
    """Internal consistency of an installed-runtime preflight: identity, pinned engine version and a build
    witness that hashes the preflight it is part of."""
    try:
        rev = plan["source_revision"]
        pinned = profiles.get(rev)
        identity = (type(v) is dict and v.get("schema") == INSTALLED_SCHEMA and v.get("status") == "PASS"
                    and v.get("failure") is None and v.get("cpu_only") is True and v.get("gpu_submitted") is False
                    and v.get("runtime_qualified") is False and v.get("run_id") == plan["run_id"]
                    and v.get("packet_sha256") == plan["packet_sha256"] and v.get("plan_sha256") == ev.digest(plan_raw)
                    and v.get("source_revision") == rev)
        if not identity:
            return False
        product, engine = v["product"], v["installed_engine"]
        installed = (product.get("sha256") == _canon_digest(product["files"]) and product["sha256"] == plan["packet_sha256"]
                     and engine.get("schema") == "sdcguard.owner-checksum-installed.v1"
                     and engine.get("source_revision") == rev and engine.get("runtime_qualified") is False
                     and engine["versions"]["vllm"] == pinned["version"])
        if not installed:
            return False
        source = v["pinned_source_guard"]
        if source.get("head") != rev or source.get("tracked_status") != "":
            return False
        mc = v["model_cache"]
        model_ok = (mc.get("model") == MODEL and mc.get("revision") == MODEL_REVISION and type(mc.get("snapshot")) is str
                    and mc["snapshot"].startswith("/") and Path(mc["snapshot"]).name == MODEL_REVISION)
        if not model_ok or not ev.same(v["python_runtime"]["identity"], engine["python_identity"]):
            return False
        w = _installed_witness(v)
        return ev.json_bytes(v["build_witness"]) == ev.json_bytes(w) and v.get("build_witness_sha256") == _canon_digest(w)
    except (ValueError, KeyError, TypeError, AttributeError):
        return False


def _source_build_ok(pre, inst, witness, payload, result, plan, plan_raw) -> bool:
    """The baseline revision's own build record: the witness hashes the installed identity, the preflight and the
    pinned source guard of this run."""
    return (witness.get("sha256") == _canon_digest(payload)
            and result.get("build_witness_sha256") == witness.get("sha256")
            and payload.get("schema") == "sdcguard.owner-checksum-build-witness.v1"
            and payload.get("installed_identity_sha256") == _canon_digest(inst)
            and payload.get("packet_sha256") == plan["packet_sha256"] and pre.get("packet_sha256") == plan["packet_sha256"]
            and pre.get("run_id") == plan["run_id"] and pre.get("status") == "PASS"
            and pre.get("schema") == "sdcguard.owner-checksum-cpu-preflight.v1"
            and inst.get("schema") == "sdcguard.owner-checksum-installed.v1" and pre.get("failure") is None
            and pre.get("plan_sha256") == ev.digest(plan_raw) and ev.same(pre.get("build_witness"), payload)
            and pre.get("build_witness_sha256") == witness.get("sha256")
            and all(pre.get(k) == payload.get(k) for k in ("build_result_sha256", "build_archive_sha256"))
            and payload.get("pinned_source_guard_sha256") == _canon_digest(pre.get("pinned_source_guard"))
            and payload.get("python_identity_sha256") == _canon_digest(pre.get("python_runtime", {}).get("identity")))


def _build_issues(preflight_raw, files, plan, result) -> tuple[list, str, str]:
    """Findings on the recorded engine build, and the (vLLM version, source revision) it names."""
    if preflight_raw is None:
        return ["recorded_engine_build_missing"], "unknown", "unknown"
    pre = ev.parse_json(preflight_raw)
    inst = pre.get("installed_engine", {})
    version = inst.get("versions", {}).get("vllm", "unknown")
    recorded = inst.get("source_revision", "unknown")
    witness = ev.object_at(files, "BUILD_WITNESS.json")
    payload = witness.get("witness", {})
    rev = plan["source_revision"]
    out = []
    if version != profiles.get(rev)["version"] or inst.get("source_revision") != rev or pre.get("source_revision") != rev:
        out.append("unsupported_recorded_engine_version")
    if pre.get("schema") == INSTALLED_SCHEMA:
        witnessed = (_installed_preflight_ok(pre, plan, files["client/REQUEST_PLAN.json"])
                     and payload.get("schema") == INSTALLED_WITNESS and ev.same(payload, pre.get("build_witness"))
                     and witness.get("sha256") == pre.get("build_witness_sha256")
                     and result.get("build_witness_sha256") == witness.get("sha256"))
        if not witnessed:
            out.append("installed_runtime_preflight_unverified")
        snap = pre.get("model_cache", {}).get("snapshot")
        for parm in plan["arms"]:
            for role in ("prefill", "decode"):
                p = parm["arm_id"] + "/" + role + "/startup-"
                starts = [ev.object_at(files, n) for n in files if n.startswith(p) and n.endswith(".json")]
                if len(starts) != 1 or type(snap) is not str or any(
                        starts[0].get(k) != snap for k in ("actual_model", "actual_tokenizer", "snapshot")):
                    out.append("installed_model_startup_binding_unverified:" + parm["arm_id"] + ":" + role)
    elif rev != profiles.BASELINE:
        out.append("candidate_requires_installed_runtime_preflight")
    elif not _source_build_ok(pre, inst, witness, payload, result, plan, files["client/REQUEST_PLAN.json"]):
        out.append("recorded_engine_build_unverified")
    return out, version, recorded


_CONSUMED = ("client/REQUEST_PLAN.json", "client/CLIENT_INVENTORY.json", "client/CLIENT_RECEIPTS.jsonl",
             "CAPTURES.json", "FINISHED.json", "BUILD_WITNESS.json")


def _run_issues(result, finished, plan, archive_raw) -> list[str]:
    out = []
    if (not ev.same(result.get("report"), finished) or result.get("archive_sha256") != ev.digest(archive_raw)
            or any(not ev.same(result.get(k), plan[k]) for k in ("run_id", "packet_sha256"))
            or any(not ev.same(finished.get(k), plan[k]) for k in ("run_id", "packet_sha256"))):
        out.append("owner_evidence_identity_disagrees")
    if not (finished.get("complete") is True and finished.get("failure") is None and finished.get("stage") == "complete"
            and finished.get("cleanup_complete") is True and finished.get("client_inventory_complete") is True):
        out.append("owner_run_completion_unverified")
    return out


def _checksum_fact(row) -> dict:
    """The checksum check of one joined request as the policy reads it."""
    calls = row["checksum_calls"]
    proof = calls[0]["conditional_scope"] if len(calls) == 1 else {}
    return dict(native_result=row["native_result"], expected_units=proof.get("expected_units"),
                compared_units=proof.get("compared_units"),
                completed=len(calls) == 1 and row["check_status"] == "passed",
                evidence_complete=row["coverage"] == "complete" and not row["reasons"],
                applicable=row["observer_enabled"],
                reason=row["reasons"][0] if row["reasons"] else "complete_recorded_comparison")


def checksum_gate(result_raw: bytes, archive_raw: bytes, preflight_raw, required, arm=None) -> dict:
    result, files = ev.parse_json(result_raw), ev.read_archive(archive_raw)
    consumed = {n: r for n, r in files.items() if n in _CONSUMED or n.endswith("/CLEANUP.json")
                or n.rsplit("/", 1)[-1].startswith(("startup-", "checksum-", "bindings-", "cache-"))}
    if preflight_raw is not None:
        consumed["CPU_PREFLIGHT.json"] = preflight_raw
    consumed["RESULT.json"] = result_raw
    ev.count_nodes(consumed, max_nodes=ev.MAX_TOTAL_JSON_NODES)
    plan = ev.object_at(files, "client/REQUEST_PLAN.json")
    captures = ev.object_at(files, "CAPTURES.json")
    report = cl.evaluate(files["client/REQUEST_PLAN.json"], files["client/CLIENT_INVENTORY.json"], files["CAPTURES.json"])
    issues = [x for x in report["hold_reasons"] if x not in cl.PROFILE_LIMITS and x != COVERAGE_HOLD]
    issues += _run_issues(result, ev.object_at(files, "FINISHED.json"), plan, archive_raw)
    build, version, recorded_rev = _build_issues(preflight_raw, files, plan, result)
    issues += build
    issues += _recording_issues(files, plan, captures)
    issues += _journal_issues(files)
    domains = {a["arm_id"]: "source_bound_candidate" if a["observer_enabled"] else "observer_disabled"
               for a in plan["arms"]}
    if any(c["qualification"] != domains.get(c["arm_id"]) for c in report["captures"]):
        issues.append("runtime_capture_source_unverified")
    rows = [dict(client_request_id=row["client_request_id"], arm_id=row["arm_id"], slot=row["slot"],
                 checks={"checksum": _checksum_fact(row)}, token_coverage=row["token_coverage"],
                 reasons=list(row["reasons"]))
            for row in report["requests"] if arm is None or row["arm_id"] == arm]
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
