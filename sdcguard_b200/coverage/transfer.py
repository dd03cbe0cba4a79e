"""`sdcguard transfer-check DIR` and `sdcguard transfer-compare BASE CAND`.

transfer-check: a separate obligation from the full-prompt gate. For each request it asks only whether the KV
chunks that actually crossed from prefill to decode (expected units from the receive plan, never from an
intersection with what was compared) were all compared by the native checksum. Statuses VERIFIED, NOT_EXERCISED
(nothing was transferred), MISMATCH, UNOBSERVABLE. The full-prompt verdict is recomputed unchanged. Exit 0 on PASS.

transfer-compare: two recordings of the same workload and configuration on two engine builds; per slot the
transfer coverage is PRESERVED, REGRESSED (a recorded native mismatch after a verified baseline) or UNVERIFIABLE.
Always exits 2: preservation of transfer coverage never overrides the full-prompt HOLD.

The statuses, reason strings and renderings keep the reference's contract (src/sdcguard/transfer_coverage.py:82-304,
transfer_upgrade.py:40-357) so the saved recordings get the same verdicts. The obligation of one request is a
short sequence of preconditions (each the only reason when it fails) and then a table of findings over a view of
its receive plan and verification record (`_TRANSFER_TABLE`); transfer-compare classifies each slot by the first
row of `_CHANGE_RULES` that applies.
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


def _seq(v) -> bool:
    return _int(v, 1, 2 ** 63 - 1)


class _Transfer:
    """One request's receive plan and verification record, read for the transfer obligation."""

    def __init__(self, plan: dict, rec: dict, prompt_tokens: int, local_tokens: int):
        self.plan, self.rec = plan, rec
        self.load, self.proof = plan["load_plan"], rec["proof"]
        self.prompt, self.local = prompt_tokens, local_tokens
        groups = self.load.get("groups")
        self.group = groups[0] if type(groups) is list and len(groups) == 1 and type(groups[0]) is dict else None

    def joined(self) -> bool:
        """plan < plan event < update < verification, and the proof names the plan and the same request."""
        pid, pev = self.plan.get("plan_sequence"), self.plan.get("sequence")
        upd, ver = self.rec.get("origin_update_sequence"), self.rec.get("sequence")
        return (all(_seq(n) for n in (pid, pev, upd, ver)) and pid < pev < upd < ver
                and type(self.proof.get("plan_sequence")) is int and self.proof["plan_sequence"] == pid
                and bool(self.plan.get("request_id")) and self.plan.get("request_id") == self.rec.get("request_id"))

    def accounting_agrees(self) -> bool:
        l = self.load
        return (type(l.get("num_tokens")) is int and l["num_tokens"] == self.prompt
                and type(l.get("num_local_computed_tokens")) is int and l["num_local_computed_tokens"] == self.local)

    def span(self):
        """The transferred chunk units the plan covers, or None when its one group does not start at the cached
        prefix and run to the end of the prompt."""
        g = self.group
        gid, size, start, count = (g.get(k) for k in ("group_id", "block_size", "start", "block_count"))
        if (not _int(gid) or not _int(size, 1) or not _int(start) or not _int(count, 1, observer.MAX_UNITS)
                or self.local % size or start != self.local // size
                or count != -(-self.prompt // size) - start):
            return None
        return [f"group:{gid}:chunk:{n}" for n in range(start, start + count)]


_TRANSFER_TABLE = (
    observer.Finding("receive_plan_to_verification_join_unverified", lambda t: not t.joined()),
    observer.Finding("planned_chunk_scope_disagrees_with_verification",
                     lambda t: not observer.plan_matches_proof(t.plan, t.proof)),
    observer.Finding("receive_plan_disagrees_with_native_cache_accounting", lambda t: not t.accounting_agrees()),
    observer.Finding("transfer_group_layout_unsupported", lambda t: t.group is None),
    observer.Finding("receive_plan_does_not_cover_transfer_span", lambda t: t.group is not None and t.span() is None),
)


def transfer_scope(plans, records, *, prompt_tokens, local_tokens, remote_tokens) -> dict:
    """Expected transfer chunks from the receive plan, compared chunks from the verification record."""
    res = dict(status="UNOBSERVABLE", reasons=[], expected_units=None, compared_units=None,
               expected_tokens=remote_tokens, compared_tokens=None, native_result="unverified", plan_sequence=None,
               update_sequence=None, verification_sequence=None)
    # what must hold before the records can be read at all; the first that fails is the only reason
    accounted = (_int(prompt_tokens, 1) and _int(local_tokens) and _int(remote_tokens)
                 and local_tokens + remote_tokens == prompt_tokens)
    if not accounted:
        res["reasons"] = ["native_transfer_token_accounting_unverified"]
        return res
    if remote_tokens == 0:
        if plans or records:
            res["reasons"] = ["zero_transfer_has_checksum_activity"]
        else:
            res.update(status="NOT_EXERCISED", expected_units=[], compared_units=[], compared_tokens=0)
        return res
    if len(plans) != 1 or len(records) != 1 or records[0].get("kind") != "verification":
        res["reasons"] = ["transfer_plan_or_verification_missing_or_ambiguous"]
        return res
    plan, rec = plans[0], records[0]
    if type(plan.get("load_plan")) is not dict or type(rec.get("proof")) is not dict:
        res["reasons"] = ["transfer_plan_metadata_missing"]
        return res
    res.update(plan_sequence=plan.get("plan_sequence"), update_sequence=rec.get("origin_update_sequence"),
               verification_sequence=rec.get("sequence"))
    t = _Transfer(plan, rec, prompt_tokens, local_tokens)
    found = observer._run(_TRANSFER_TABLE, t)
    expected = t.span() if t.group is not None else None
    d = observer.classify_verification(rec, max_units=observer.MAX_UNITS)
    found += [r for r in d["reasons"] if r != observer.CACHED_PREFIX_REASON]
    if not expected or d["compared_units"] != expected:
        found.append("transfer_comparison_scope_incomplete")
    if d["native_result"] == "mismatch":
        found.append("native_checksum_mismatch")
    elif d["native_result"] != "passed" or rec.get("native_return") is not True:
        found.append("native_passing_checksum_not_recorded")
    res.update(expected_units=expected, native_result=d["native_result"], compared_units=d["compared_units"],
               reasons=_uniq(found))
    if not found:
        res.update(status="VERIFIED", compared_tokens=remote_tokens)
    elif d["native_result"] == "mismatch":
        res["status"] = "MISMATCH"
    return res


# findings that may accompany an exercised-nothing request without making it unobservable
_NOT_EXERCISED_OK = {"unambiguous_active_checksum_recorder_missing", "client_to_native_request_join_unverified"}


class _Recording:
    """A recording's files as the transfer obligation reads them: the full-prompt verdict, the client join, the
    per-arm cache accounting and checksum records."""

    def __init__(self, result_raw, archive_raw, preflight_raw):
        self.full = gate.checksum_gate(result_raw, archive_raw, preflight_raw, ["checksum"])
        files = ev.read_archive(archive_raw)
        self.plan = ev.object_at(files, "client/REQUEST_PLAN.json")
        self.inventory = ev.object_at(files, "client/CLIENT_INVENTORY.json")
        self.captures = ev.object_at(files, "CAPTURES.json")["captures"]
        self.joined = cl.evaluate(files["client/REQUEST_PLAN.json"], files["client/CLIENT_INVENTORY.json"],
                                  files["CAPTURES.json"])
        self.cache = {}
        cached = self.plan.get("prefix_caching") is True
        for arm in self.plan["arms"]:
            mine = [c for c in self.captures if c.get("arm_id") == arm["arm_id"]]
            if arm["observer_enabled"] and len(mine) == 1 and cached:
                self.cache[arm["arm_id"]] = cl.cache_facts(mine[0], self.plan, arm)

    def stray_records(self) -> int:
        """Checksum records of the captures that no joined request owns."""
        known = {(r["arm_id"], r["internal_request_id"]) for r in self.joined["requests"]
                 if type(r["internal_request_id"]) is str}
        return sum(1 for cap in self.captures for snap in cap.get("checksum_snapshots", [])
                   for rec in snap.get("records", [])
                   if type(rec) is not dict or (cap["arm_id"], rec.get("request_id")) not in known)

    def records_of(self, row) -> list:
        mine = [c for c in self.captures if c.get("arm_id") == row["arm_id"]]
        snaps = mine[0].get("checksum_snapshots", []) if len(mine) == 1 else []
        internal = row["internal_request_id"]
        return [r for s in snaps for r in s.get("records", []) if type(r) is dict and type(internal) is str
                and r.get("request_id") == internal]

    def request(self, row) -> dict:
        """The transfer verdict of one joined request (before the recording-wide reasons are added)."""
        errors = [reason for reason, bad in (("client_request_completion_unverified", row["client_status"] != "complete"),
                                             ("client_to_native_request_join_unverified", row["binding_status"] != "matched"),
                                             ("observer_disabled", not row["observer_enabled"])) if bad]
        raws = [r for r in self.inventory["requests"] if type(r) is dict and r.get("arm_id") == row["arm_id"]
                and r.get("slot") == row["slot"]]
        facts, acct = self.cache.get(row["arm_id"]), {}
        if facts is None or len(raws) != 1:
            errors.append("native_cache_accounting_unavailable")
        else:
            acct, cerr = cl.cache_usage(facts, raws[0], row, for_transfer=True)
            errors += cerr
        recs = self.records_of(row)
        dec, pre = acct.get("decode", {}), acct.get("prefill", {})
        local, remote = dec.get("num_local_cached_tokens"), dec.get("num_external_cached_tokens")
        scoped = transfer_scope([r for r in recs if r.get("kind") == "recv_plan"],
                                [r for r in recs if r.get("kind") != "recv_plan"],
                                prompt_tokens=row["prompt_tokens"], local_tokens=local, remote_tokens=remote)
        if dec.get("num_computed_tokens") != 0:
            errors.append("locally_computed_prompt_scope_unsupported")
        if len(acct) != 2:
            errors.append("both_native_cache_accounts_required")
        errors += [x for call in row["checksum_calls"] for x in call["recording_issues"]]
        errors += [x for cap in self.joined["captures"] if cap["arm_id"] == row["arm_id"] for x in cap["issues"]]
        status = scoped["status"]
        if errors and (status != "NOT_EXERCISED" or set(errors) - _NOT_EXERCISED_OK):
            status = "UNOBSERVABLE"
        return dict(client_request_id=row["client_request_id"], arm_id=row["arm_id"], slot=row["slot"],
                    internal_request_id=row["internal_request_id"], status=status,
                    reasons=_uniq(errors + scoped["reasons"]), comparison=scoped,
                    tokens=dict(prompt=row["prompt_tokens"], expected_transfer=remote,
                                compared_transfer=scoped["compared_tokens"] if not errors else None,
                                decode_cache_outside_transfer=local,
                                prefill_cache_reused=pre.get("num_local_cached_tokens")))


def _decision(row) -> str:
    if row["reasons"] or row["status"] not in ("VERIFIED", "NOT_EXERCISED"):
        return "HOLD"
    return "NOT_EXERCISED" if row["status"] == "NOT_EXERCISED" else "PASS"


def _total(rows, name):
    vals = [r["tokens"][name] for r in rows]
    return sum(vals) if vals and all(type(v) is int for v in vals) else None


def evaluate(result_raw, archive_raw, preflight_raw) -> dict:
    rec = _Recording(result_raw, archive_raw, preflight_raw)
    issues = [r for r in rec.full["hold_reasons"] if r != gate.COVERAGE_HOLD]
    if rec.plan.get("prefix_caching") is not True:
        issues.append("transfer_profile_requires_native_cache_accounting")
    issues += ["unjoined_native_transfer_record"] * rec.stray_records()
    rows = [rec.request(row) for row in rec.joined["requests"]]
    issues += [x for f in rec.cache.values() for x in cl.unexpected_cache(f)]
    issues = _uniq(issues)
    for row in rows:
        row["reasons"] = _uniq(row["reasons"] + issues)
        row["decision"] = _decision(row)
    counts = Counter(r["status"] for r in rows)
    if not rows or not counts["VERIFIED"]:
        issues.append("no_verified_transfer_requests")
    if any(r["decision"] == "HOLD" for r in rows):
        issues.append("transfer_comparison_obligation_incomplete")
    exp = [r["comparison"]["expected_units"] for r in rows]
    exp_n = sum(len(u) for u in exp) if exp and all(type(u) is list for u in exp) else None
    full = rec.full
    return dict(schema=SCHEMA, owner=OWNER, scope=SCOPE, transfer_decision="HOLD" if issues else "PASS",
                release_decision=full["decision"], full_prompt_gate=full, runtime_qualified=False, engine=full["engine"],
                inputs_sha256=dict(result=ev.digest(result_raw), archive=ev.digest(archive_raw),
                                   preflight=ev.digest(preflight_raw) if preflight_raw is not None else None),
                summary=dict(planned_requests=len(rows), verified_requests=sum(r["decision"] == "PASS" for r in rows),
                             not_exercised_requests=counts["NOT_EXERCISED"],
                             held_requests=sum(r["decision"] == "HOLD" for r in rows), statuses=dict(counts),
                             expected_chunk_positions=exp_n, prompt_tokens=_total(rows, "prompt"),
                             expected_transfer_tokens=_total(rows, "expected_transfer"),
                             compared_transfer_tokens=_total(rows, "compared_transfer"),
                             decode_cached_tokens_outside_transfer=_total(rows, "decode_cache_outside_transfer")),
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
    if not all(out.values()):
        raise ev.EvidenceError("engine identity is incomplete")
    return out


_VERSION_TEXT = re.compile(r"[0-9][0-9A-Za-z.+_-]{0,127}")
_RUNTIME_PACKAGES = {"vllm", "torch", "triton", "nixl", "nixl-cu12", "nixl-cu13"}


def _runtime_identity(pre):
    inst = pre["installed_engine"]
    py, vers = inst["python_identity"], inst["versions"]
    ver = py.get("version")
    versions_ok = (type(vers) is dict and _RUNTIME_PACKAGES <= vers.keys()
                   and all(type(v) is str and _VERSION_TEXT.fullmatch(v) for k, v in vers.items() if k != "uv"))
    python_ok = (py.get("implementation") == "cpython" and py.get("platform") == "linux"
                 and py.get("soabi") == "cpython-312-x86_64-linux-gnu" and type(ver) is list and len(ver) == 3
                 and all(type(n) is int and 0 <= n <= 999 for n in ver) and ver[:2] == [3, 12])
    if not (versions_ok and python_ok):
        raise ev.EvidenceError("recorded runtime identity is missing, unknown or unsupported")
    return dict(versions={k: v for k, v in vers.items() if k != "uv"},
                python={k: py[k] for k in ("implementation", "version", "platform", "soabi")})


def _client_input(stage) -> dict:
    """What a client stage asked, without the per-run identities (request ids, transfer handles)."""
    body = _without(stage["request_body"], {"request_id", "kv_transfer_params"})
    body["kv_transfer_params"] = _without(stage["request_body"]["kv_transfer_params"], _TRANSFER_VOLATILE)
    return dict(method=stage["method"], path=stage["path"], body_sha256=_h(body),
                headers_sha256=_h(_without(stage["request_headers"], {"X-Request-Id"})))


def _workload(plan, inventory) -> tuple[dict, dict]:
    """The planned workload without run identities, and the digest of every slot's request spec (plan fields
    plus what the client actually sent)."""
    raw_rows = _index(inventory["requests"])
    work = _without(plan, {"run_id", "packet_sha256", "source_revision", "arms"})
    work["arms"] = []
    slots = {}
    for arm in plan["arms"]:
        norm = _without(arm, {"engine_session_id", "requests"})
        norm["requests"] = []
        for r in arm["requests"]:
            k = _key(dict(arm_id=arm["arm_id"], slot=r["slot"]))
            if k in slots:
                raise ev.EvidenceError("duplicate planned comparison slot")
            raw = raw_rows.get(k)
            if raw is None:
                raise ev.EvidenceError("client input missing from comparison slot")
            spec = _without(r, {"client_request_id", "prefill_request_id"})
            spec["client_inputs"] = {role: _client_input(raw[role]) for role in ("prefill", "decode")}
            slots[k] = _h(spec)
            norm["requests"].append(spec)
        work["arms"].append(norm)
    if set(raw_rows) != set(slots):
        raise ev.EvidenceError("client inventory and planned comparison slots differ")
    return work, slots


def _engine_configs(plan, captures) -> tuple[list, list]:
    """(engine sessions, each engine's recorded startup configuration without per-run identities)."""
    sessions, configs = [], []
    for cap in captures:
        sess = cap["engine_session_id"]
        if type(sess) is not str or not sess:
            raise ev.EvidenceError("engine session missing")
        sessions.append(sess)
        for role, v in (("decode", cap), ("prefill", cap["prefill_capture"])):
            st = v["startup"]
            if not _REQUIRED_CONFIG <= st.keys():
                raise ev.EvidenceError("recorded comparison configuration is incomplete")
            cfg = _without(st, _STARTUP_VOLATILE)
            # the baseline revision's recorder names a setting its source does not have; it is off there
            if plan["source_revision"] == profiles.BASELINE and cfg.get("defer_async_loads") == "not_in_source_profile":
                cfg["defer_async_loads"] = False
            configs.append(dict(arm_id=cap["arm_id"], role=role, config=cfg))
    return sessions, configs


def _contracts(files, pre) -> dict:
    plan = ev.object_at(files, "client/REQUEST_PLAN.json")
    work, slots = _workload(plan, ev.object_at(files, "client/CLIENT_INVENTORY.json"))
    sessions, configs = _engine_configs(plan, ev.object_at(files, "CAPTURES.json")["captures"])
    model = pre["model_cache"]
    if not all(model.get(k) for k in ("model", "revision", "files")):
        raise ev.EvidenceError("model and tokenizer file identities are missing")
    runtime = _runtime_identity(pre)
    runtime["versions"].pop("vllm")            # the engine version is what the comparison is about
    conf = dict(engines=configs, model={k: model[k] for k in ("model", "revision", "files")}, runtime=runtime)
    return dict(workload_sha256=_h(work), config_sha256=_h(conf), slots=slots, sessions=sorted(sessions),
                run_id=plan["run_id"])


# hold reasons of a side's transfer check that only say coverage is incomplete (what the comparison is about)
_COVERAGE_ONLY = {"required_checksum_coverage_incomplete", "transfer_comparison_obligation_incomplete",
                  "no_verified_transfer_requests"}


def _side(raw) -> dict:
    hashes = {k: ev.digest(v) if v is not None else None for k, v in zip(("result", "archive", "preflight"), raw)}
    side = dict(inputs_sha256=hashes, errors=[], assessment=None, contracts=None, engine_identity_sha256=None)
    try:
        side["assessment"] = evaluate(*raw)
        pre = ev.parse_json(raw[2]) if raw[2] is not None else {}
        side["contracts"] = _contracts(ev.read_archive(raw[1]), pre)
        gaps = [r for r in side["assessment"]["hold_reasons"] if r not in _COVERAGE_ONLY]
        side["errors"] += ["input_qualification:" + r for r in gaps]
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


_EXERCISE = ("prompt", "expected_transfer", "decode_cache_outside_transfer", "prefill_cache_reused")


def _scope_known(row) -> bool:
    units = row["comparison"]["expected_units"]
    return all(type(row["tokens"][k]) is int for k in _EXERCISE) and type(units) is list and bool(units)


def _same_exercise(b, a) -> bool:
    return (all(b["tokens"][k] == a["tokens"][k] for k in _EXERCISE)
            and b["comparison"]["expected_units"] == a["comparison"]["expected_units"])


def _recorded_mismatch(a) -> bool:
    """The candidate's comparison ran over the whole transfer and the engine reported a mismatch: nothing else
    held it."""
    c = a["comparison"]
    return (a["status"] == "MISMATCH" and c["native_result"] == "mismatch"
            and set(a["reasons"]) == {"native_checksum_mismatch"} and set(c["reasons"]) == {"native_checksum_mismatch"}
            and c["compared_units"] == c["expected_units"])


# (applies to (before, after, comparable, same_slot), change, reason); the first rule that applies decides
_CHANGE_RULES = (
    (lambda b, a, ok, same: not ok or not same, "UNVERIFIABLE", "workload_or_configuration_not_comparable"),
    (lambda b, a, ok, same: b is None or a is None, "UNVERIFIABLE", "request_missing_from_one_side"),
    (lambda b, a, ok, same: b["decision"] != "PASS", "UNVERIFIABLE", "baseline_transfer_not_verified"),
    (lambda b, a, ok, same: not (_scope_known(b) and _scope_known(a)), "UNVERIFIABLE", "transfer_scope_unverifiable"),
    (lambda b, a, ok, same: not _same_exercise(b, a), "UNVERIFIABLE", "transfer_exercise_changed"),
    (lambda b, a, ok, same: a["decision"] != "PASS" and _recorded_mismatch(a), "REGRESSED",
     "candidate_recorded_native_mismatch"),
    (lambda b, a, ok, same: a["decision"] != "PASS", "UNVERIFIABLE", "candidate_transfer_evidence_unverifiable"),
)


def _change(before, after, comparable, same_slot):
    for applies, change, reason in _CHANGE_RULES:
        if applies(before, after, comparable, same_slot):
            return change, [reason]
    return "PRESERVED", []


def _build_relation(base, cand) -> str:
    bi, ci = base["engine_identity_sha256"], cand["engine_identity_sha256"]
    if bi is None or ci is None:
        return "unknown"
    return "same_recorded_build" if bi == ci else "different_recorded_build"


def _recording_relation(base, cand) -> str:
    if base["inputs_sha256"] == cand["inputs_sha256"]:
        return "same_evidence"
    b, c = base["contracts"], cand["contracts"]
    if b is None or c is None or base["errors"] or cand["errors"]:
        return "unknown"
    independent = b["run_id"] != c["run_id"] and not set(b["sessions"]) & set(c["sessions"])
    return "distinct_recorded_sessions" if independent else "overlapping_recording_identity"


def _slot_rows(base, cand, comparable) -> list:
    b, c = base["contracts"], cand["contracts"]
    before = _index(base["assessment"]["requests"]) if base["assessment"] else {}
    after = _index(cand["assessment"]["requests"]) if cand["assessment"] else {}
    rows = []
    for k in sorted(before.keys() | after.keys()):
        left, right = before.get(k), after.get(k)
        same_slot = b is not None and c is not None and k in b["slots"] and b["slots"].get(k) == c["slots"].get(k)
        change, why = _change(left, right, comparable, same_slot)
        lost = bool(left and left["decision"] == "PASS" and (not right or right["decision"] != "PASS"))
        rows.append(dict(arm_id=k[0], slot=k[1], coverage_change=change, reasons=why, lost_passing_evidence=lost,
                         baseline=_row_view(left), candidate=_row_view(right)))
    return rows


def compare(baseline_raw, candidate_raw) -> dict:
    base, cand = _side(baseline_raw), _side(candidate_raw)
    b, c = base["contracts"], cand["contracts"]
    errors = [f"{lab}:{e}" for lab, side in (("baseline", base), ("candidate", cand)) for e in side["errors"]]
    both = b is not None and c is not None
    if not (both and b["workload_sha256"] == c["workload_sha256"]):
        errors.append("workload_not_comparable")
    if not (both and b["config_sha256"] == c["config_sha256"]):
        errors.append("configuration_not_comparable")
    comparable = not errors
    build, relation = _build_relation(base, cand), _recording_relation(base, cand)
    rows = _slot_rows(base, cand, comparable)
    counts = Counter(r["coverage_change"] for r in rows)
    assessments = {"baseline": base["assessment"], "candidate": cand["assessment"]}
    revisions = tuple(a["engine"].get("source_revision") if a else None for a in assessments.values())
    transition = revisions == (profiles.BASELINE, profiles.CANDIDATE) and comparable
    holds = list(errors)
    holds += [reason for reason, bad in (
        ("recorded_native_comparison_regressed", bool(counts["REGRESSED"])),
        ("coverage_preservation_unverifiable", bool(counts["UNVERIFIABLE"]) or not rows),
        ("independent_recordings_not_established", relation != "distinct_recorded_sessions"),
        ("changed_engine_build_not_established", build != "different_recorded_build")) if bad]
    for lab, a in assessments.items():
        if a is None or a["transfer_decision"] != "PASS":
            holds.append(lab + "_transfer_check_held")
        if a is None or a["release_decision"] != "PASS":
            holds.append(lab + "_full_prompt_policy_held")
    if not transition:
        holds.append("changed_build_transition_not_qualified")
    preserved = (transition and relation == "distinct_recorded_sessions" and build == "different_recorded_build"
                 and bool(rows) and counts["PRESERVED"] == len(rows)
                 and all(a["transfer_decision"] == "PASS" for a in assessments.values()))
    return dict(schema=UP_SCHEMA, owner=OWNER, policy=POLICY, scope=SCOPE, upgrade_decision="HOLD",
                transfer_preservation_decision="PASS" if preserved else "HOLD",
                runtime_upgrade_witness="distinct source-bound recordings" if preserved else "not established",
                comparison_status="COMPARABLE" if comparable else "UNVERIFIABLE", build_relation=build,
                recording_relation=relation,
                summary=dict(compared_slots=len(rows), preserved=counts["PRESERVED"], regressed=counts["REGRESSED"],
                             unverifiable=counts["UNVERIFIABLE"],
                             lost_passing_evidence=sum(r["lost_passing_evidence"] for r in rows)),
                baseline=_view(base), candidate=_view(cand), requests=rows, hold_reasons=_uniq(holds),
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
