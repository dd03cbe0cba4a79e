"""The supervised coverage capture (`sdcguard operator`) on the CPU: preflight refusals, the supervisor's cleanup
evidence for a recorder that finishes, fails or overruns its deadline (its whole process group killed), and a
failed run recorded as HOLD."""
import json
import sys

from sdcguard_b200.serve import operator as op


def test_preflight_refuses_existing_output_and_missing_gpus(tmp_path):
    r = op.preflight(tmp_path)                     # exists
    assert r["status"] == "FAIL" and "output_is_new" in r["failure"]
    r = op.preflight(tmp_path / "new", gpus=64)
    assert r["status"] == "FAIL" and "gpus_visible" in r["failure"]
    assert r["build"].get("sources_digest")


def test_supervisor_clean_failed_and_deadline(tmp_path):
    ok = op.supervise([sys.executable, "-c", "print('hi')"], tmp_path / "a.log", 30)
    assert ok["clean"] and ok["exit_code"] == 0 and not ok["timed_out"]
    bad = op.supervise([sys.executable, "-c", "raise SystemExit(3)"], tmp_path / "b.log", 30)
    assert not bad["clean"] and bad["exit_code"] == 3
    # a recorder that forks a child and hangs: the deadline kills the whole group
    code = "import subprocess, sys, time; subprocess.Popen([sys.executable, '-c', 'import time; time.sleep(60)']); time.sleep(60)"
    slow = op.supervise([sys.executable, "-c", code], tmp_path / "c.log", 2)
    assert slow["timed_out"] and not slow["clean"] and not slow["group_left_running"]


def test_run_records_hold(tmp_path, monkeypatch, capsys):
    out = tmp_path / "cap"
    monkeypatch.setattr(op, "preflight", lambda o, gpus=1: {"status": "PASS", "failure": None,
                                                             "checks": {"output_is_new": True}})
    monkeypatch.setattr(op, "supervise", lambda cmd, log, deadline: {"clean": False, "exit_code": 1,
                                                                     "timed_out": False, "group_left_running": False})
    rc = op.main(["run", "--out", str(out), "--require", "checksum"])
    assert rc == 2
    err = json.loads((out / "OPERATOR_ERROR.json").read_text())
    assert err["decision"] == "HOLD" and (out / "SUPERVISOR.json").exists()
    assert op.main(["run", "--out", str(tmp_path / "x"), "--require", "lease"]) == 2
    monkeypatch.undo()
    assert op.main(["run", "--out", str(out), "--require", "checksum"]) == 2      # output exists
