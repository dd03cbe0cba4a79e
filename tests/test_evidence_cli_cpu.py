"""The evidence commands through the `sdcguard` command line (exit codes and files), on CPU: config-safety,
evidence build / report-verify, upgrade, record-plan, operator-setup, model-ref, regression, lifetime."""
import json

from sdcguard_b200 import cli
from sdcguard_b200.evidence import operator_setup


def _dep(tmp_path, **over):
    d = json.loads(json.dumps(operator_setup.TEMPLATE))
    for w in d["workers"]:
        w["version"], w["build"] = "0.1.0", "abc"
        (tmp_path / w["startup_log"]).write_text(f"sdcguard_b200 engine: kv_pages={w['kv_pages']} page_tokens=16\n")
    d["workers"][0].update(over)
    p = tmp_path / ("dep_%d.json" % len(over))
    p.write_text(json.dumps(d))
    return str(p)


def test_config_safety_report_and_upgrade_exit_codes(tmp_path, capsys):
    good, bad = _dep(tmp_path), _dep(tmp_path, release="early")
    assert cli.main(["config-safety", good]) == 0
    assert cli.main(["config-safety", bad]) == 3
    cg, cb = tmp_path / "cg.json", tmp_path / "cb.json"
    for dep, out in ((good, cg), (bad, cb)):
        capsys.readouterr()
        cli.main(["config-safety", dep, "--json"])
        out.write_text(capsys.readouterr().out)
    rg, rb = tmp_path / "rg.json", tmp_path / "rb.json"
    assert cli.main(["evidence", "build", str(rg), "--section", f"config={cg}"]) == 0
    assert cli.main(["evidence", "build", str(rb), "--section", f"config={cb}"]) == 0
    assert cli.main(["report-verify", str(rg)]) == 0
    env = json.loads(rg.read_text())
    env["findings"][next(iter(env["findings"]))]["verdict"] = "violated"
    (tmp_path / "tampered.json").write_text(json.dumps(env))
    assert cli.main(["report-verify", str(tmp_path / "tampered.json")]) == 1
    assert cli.main(["upgrade", str(rg), str(rg)]) == 0
    assert cli.main(["upgrade", str(rg), str(rb)]) == 3


def test_record_plan_setup_model_ref_regression_lifetime(tmp_path):
    dep = _dep(tmp_path)
    assert cli.main(["record-plan", dep, "--out", str(tmp_path / "plan.json")]) == 0
    assert "pd_mp" in json.loads((tmp_path / "plan.json").read_text())["launch_shell"]
    assert cli.main(["operator-setup", "export", str(tmp_path / "setup")]) == 0
    assert cli.main(["operator-setup", "verify", str(tmp_path / "setup")]) == 0
    m = tmp_path / "model"
    m.mkdir()
    (m / "w.bin").write_bytes(b"\x00" * 64)
    assert cli.main(["model-ref", "capture", str(m), "--out", str(tmp_path / "ref.json")]) == 0
    assert cli.main(["model-ref", "observe", str(tmp_path / "ref.json"), str(m)]) == 0
    (m / "w.bin").write_bytes(b"\x01" * 64)
    assert cli.main(["model-ref", "observe", str(tmp_path / "ref.json"), str(m)]) == 1
    assert cli.main(["regression", "run"]) == 0
    assert cli.main(["regression", "export", str(tmp_path / "case")]) == 0
    assert cli.main(["regression", "verify", str(tmp_path / "case")]) == 0
    assert cli.main(["lifetime", "conformance"]) == 0


def test_inventory_overhead_assignment_forward_cli(tmp_path):
    from sdcguard_b200.coverage import evidence as ev
    from sdcguard_b200.evidence import inventory
    from sdcguard_b200.lifetime import conformance
    rec = tmp_path / "rec"
    rec.mkdir()
    prompts = {"e1": [1, 2, 3], "e2": [5, 6]}
    (rec / "REQUEST_PLAN.json").write_text(json.dumps({"requests": [
        {"request_id": r, "prompt_tokens": len(t), "prompt_sha256": ev.digest(ev.json_bytes(t))}
        for r, t in prompts.items()]}))
    (rec / "OBSERVER.json").write_text(json.dumps({"records": [{"request_id": r} for r in prompts]}))
    inv = tmp_path / "inv.json"
    inv.write_text(json.dumps(inventory.from_prompts({"c1": [1, 2, 3], "c2": [5, 6]})))
    assert cli.main(["inventory", str(inv), str(rec)]) == 0
    line = {"metric": "m", "n_gpus": 1, "dtype": "bf16", "config": {"a": 1}, "unit": "tok/s"}
    (tmp_path / "on.jsonl").write_text(json.dumps(dict(line, value=98.0)) + "\n")
    (tmp_path / "off.jsonl").write_text(json.dumps(dict(line, value=100.0)) + "\n")
    assert cli.main(["overhead", "compare", "--on", str(tmp_path / "on.jsonl"), "--off", str(tmp_path / "off.jsonl"),
                     "--bound", "3"]) == 0
    assert cli.main(["overhead", "compare", "--on", str(tmp_path / "on.jsonl"), "--off", str(tmp_path / "off.jsonl"),
                     "--bound", "1"]) == 3
    with conformance.cpu_transfers():
        events = conformance._scenario("prefix_reuse")
    ev_path = tmp_path / "lifetime.jsonl"
    ev_path.write_text("".join(json.dumps(e) + "\n" for e in events))
    assert cli.main(["assignment", "inspect", str(ev_path)]) == 0
    assert cli.main(["forward-inputs", "inspect", str(ev_path)]) == 0
    assert cli.main(["forward-inputs", "packet", str(ev_path), "--out", str(tmp_path / "fp.json")]) == 0
    assert cli.main(["forward-inputs", "verify", str(tmp_path / "fp.json")]) == 0
