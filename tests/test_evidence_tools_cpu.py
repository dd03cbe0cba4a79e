"""Offline evidence tools: static deployment contracts, the report envelope and its verification, the upgrade
preservation policy, client-inventory join, matched-run overhead with identity, model file binding, recorded page
assignment and forward inputs (from the CPU conformance run of pd.py), the recording plan, operator setup and the
saved regression case. Everything here runs on the CPU and starts no engine."""
import json
import os

import pytest

from sdcguard_b200.evidence import (assignment, catalog, config, forward, inventory, model_reference, operator_setup,
                                    overhead, recording_plan, regression, report, upgrade)


def _deployment(tmp_path, name="dep.json", **over):
    d = json.loads(json.dumps(operator_setup.TEMPLATE))
    for w in d["workers"]:
        w["version"], w["build"] = "0.1.0", "abc"
        (tmp_path / w["startup_log"]).write_text(
            f"boot\nsdcguard_b200 engine: engine=sdcguard_b200 kv_pages={w['kv_pages']} page_tokens=16 checked=True\n")
    for k, v in over.items():
        d["workers"][0][k] = v
    p = tmp_path / name
    p.write_text(json.dumps(d))
    return str(p)


def test_config_contracts_pass_then_fail_on_unsafe_settings(tmp_path):
    doc, prov = config.load_deployment(_deployment(tmp_path))
    a = config.assess(doc, prov)
    assert a["verdict"] == "PASS", config.render(a)
    for w in a["workers"]:
        for r in w["rules"]:
            assert catalog.validate_finding(r) == []
    doc, prov = config.load_deployment(_deployment(tmp_path, release="early", checked=False, kv_pages=10))
    a = config.assess(doc, prov)
    bad = {r["id"] for r in a["workers"][0]["rules"] if r["verdict"] == "violated"}
    assert a["verdict"] == "FAIL" and {"protection.deferred_release", "protection.gemm_abft",
                                       "capacity.planned"} <= bad


def test_config_missing_facts_are_unknown_not_satisfied(tmp_path):
    p = _deployment(tmp_path, startup_log="nope.log")
    doc, prov = config.load_deployment(p)
    del doc["workers"][1]["kv_checksums"]
    a = config.assess(doc, prov)
    r0 = {r["id"]: r["verdict"] for r in a["workers"][0]["rules"]}
    r1 = {r["id"]: r["verdict"] for r in a["workers"][1]["rules"]}
    assert r0["capacity.startup"] == "unknown" and r1["protection.kv_checksum"] == "unknown"
    assert a["verdict"] == "HOLD"


def test_report_envelope_verifies_and_detects_tampering(tmp_path):
    doc, prov = config.load_deployment(_deployment(tmp_path))
    env = report.build({"config": config.assess(doc, prov)})
    assert report.verify(env) == [] and env["counts"]["satisfied"] > 5
    assert "config/prefill0/protection.kv_checksum" in env["findings"]
    env2 = json.loads(json.dumps(env))
    env2["findings"]["config/prefill0/protection.kv_checksum"]["verdict"] = "violated"
    assert report.verify(env2)


def test_upgrade_policy_classifies(tmp_path):
    doc, prov = config.load_deployment(_deployment(tmp_path))
    before = report.build({"config": config.assess(doc, prov)})
    same = upgrade.compare(before, before)
    assert same["verdict"] == "PRESERVED"
    doc, prov = config.load_deployment(_deployment(tmp_path, release="early"))
    after = report.build({"config": config.assess(doc, prov)})
    c = upgrade.compare(before, after)
    assert c["verdict"] == "REGRESSED" and c["counts"]["regressed"] >= 1
    assert upgrade.verify_comparison(c, before, after) == []


def _recording(tmp_path, prompts):
    from sdcguard_b200.coverage import evidence as ev
    d = tmp_path / "rec"
    d.mkdir()
    plan = {"requests": [{"request_id": rid, "prompt_tokens": len(t), "prompt_sha256": ev.digest(ev.json_bytes(t))}
                         for rid, t in prompts.items()]}
    obs = {"records": [{"request_id": rid, "kind": "verification"} for rid in prompts]}
    (d / "REQUEST_PLAN.json").write_text(json.dumps(plan))
    (d / "OBSERVER.json").write_text(json.dumps(obs))
    return str(d)


def test_inventory_join_complete_and_ambiguous(tmp_path):
    prompts = {"e1": [1, 2, 3], "e2": [4, 5, 6, 7]}
    rec = _recording(tmp_path, prompts)
    inv = inventory.from_prompts({"c1": [1, 2, 3], "c2": [4, 5, 6, 7]})
    r = inventory.reconcile(inv, rec)
    assert r["status"] == "complete" and r["matched_requests"] == 2
    inv2 = inventory.from_prompts({"c1": [1, 2, 3]})
    r2 = inventory.reconcile(inv2, rec)
    assert r2["status"] == "unknown" and r2["unexpected"] == [{"request": "e2",
                                                              "reason": "transfer outside the declared batch"}]


def test_overhead_summary_and_identity(tmp_path):
    cfg = {"model": "m", "global_batch": 8}
    line = {"metric": "tok/s", "n_gpus": 1, "dtype": "bf16", "config": cfg, "unit": "tokens/s"}
    on = [dict(line, value=v) for v in (97.0, 98.0)]
    off = [dict(line, value=v) for v in (100.0, 100.5)]
    ident = overhead.prepare_identity(cfg, None, "GPU-00000000-1111-2222-3333-444444444444")
    r = overhead.summarize(on, off, bound_pct=3.0, identity=ident)
    assert r["verdict"] == "PASS" and 1.5 < r["overhead_pct"] < 3.0
    r = overhead.summarize(on, [dict(off[0], n_gpus=2)], identity=ident)
    assert r["verdict"] == "HOLD" and "runs differ in n_gpus" in r["issues"]


def test_model_reference_capture_and_observe(tmp_path):
    m = tmp_path / "model"
    m.mkdir()
    (m / "w.bin").write_bytes(b"\x01" * 100)
    (m / "config.json").write_text("{}")
    ref = model_reference.bind(model_reference.capture(str(m)), "tiny")
    assert model_reference.observe(ref, str(m))["match"]
    (m / "w.bin").write_bytes(b"\x02" * 100)
    r = model_reference.observe(ref, str(m))
    assert not r["match"] and r["changed"] == ["w.bin"]


def test_assignment_and_forward_reports_from_conformance_events():
    from sdcguard_b200.lifetime import conformance
    with conformance.cpu_transfers():
        ev = conformance._scenario("prefix_reuse")
    a = assignment.inspect_payload(ev)
    f = forward.inspect_payload(ev)
    assert a["verdict"] == "PASS" and f["verdict"] == "PASS" and f["forward_passes"] == 16
    pkt = json.loads(json.dumps(forward.create_packet(ev)))
    assert forward.verify_packet(pkt) == []
    # a forward pass naming a page of another request is reported
    bad = [dict(e) for e in ev]
    i = next(k for k, e in enumerate(bad) if e["ev"] == "forward" and e["phase"] == "decode")
    other = next(e for e in bad[:i] if e["ev"] == "alloc" and e["region"][0] == "decode"
                 and e["owner"] != bad[i]["request"])
    bad[i] = dict(bad[i], regions=[[other["region"][0], other["region"][1], 1]] + bad[i]["regions"][1:])
    assert forward.inspect_payload(bad)["verdict"] == "FAIL"
    dbl = ev[:1] + [dict(ev[0], owner="intruder")]
    assert assignment.inspect_payload(dbl)["verdict"] == "FAIL"


def test_recording_plan_and_operator_setup(tmp_path):
    dep = _deployment(tmp_path)
    doc, prov = config.load_deployment(dep)
    plan = recording_plan.prepare_recording_plan(doc, prov, out_dir=str(tmp_path / "rec"))
    assert "sdcguard_b200.serve.pd_mp" in plan["launch"] and "--verify-cached-prefix" in plan["launch"]
    doc2, prov2 = config.load_deployment(_deployment(tmp_path, "unsafe.json", release="early"))
    with pytest.raises(ValueError):
        recording_plan.prepare_recording_plan(doc2, prov2)
    out = tmp_path / "setup"
    operator_setup.export_setup(str(out))
    assert operator_setup.verify_output(str(out)) == []
    (out / "recording.env.json").write_text("{}")
    assert operator_setup.verify_output(str(out))
    assert operator_setup.preflight(dep)["ok"]


def test_regression_case_runs_and_bundle_verifies(tmp_path):
    for v in ("buggy", "fixed"):
        assert regression.judge(regression.run_case(v), v)["status"] == "pass"
    out = tmp_path / "case"
    regression.export_case(str(out))
    assert regression.verify_bundle(str(out)) == []
    r = json.loads((out / "RESULT_fixed.json").read_text())
    r["findings"] = [{"rule": "R2"}]
    (out / "RESULT_fixed.json").write_text(json.dumps(r))
    assert regression.verify_bundle(str(out))
