"""Upgrade gate of library GEMMs on the CPU: capture a case, run it in a fresh process, and the verdict rules
(PASSED / REGRESSED / UNCHANGED / FIXED / INCONCLUSIVE, exit codes) on constructed run records."""
import json
import os

import pytest

from sdcguard_b200.tools import upgrade_gate as ug


def _run(wrong, n=20, kernels=("k1",), cond=None, log=True):
    runs = [{"wrong": 1 if i < wrong else 0, "unwritten": 0} for i in range(n)]
    c = cond or {"gpu_name": "B200", "compute_capability": "10.0", "sms_visible": 148, "device_type": "cuda",
                 "env": {}, "matmul": {"tf32": False}}
    return {"runs": runs, "n": n, "conditions": c,
            "kernel_log": {"log": log, "kernels": {k: n for k in kernels}}}


def test_verdicts():
    assert ug.verdict(_run(0), _run(0))["verdict"] == "PASSED"
    assert ug.verdict(_run(0), _run(2))["verdict"] == "REGRESSED"
    assert ug.verdict(_run(5), _run(3))["verdict"] == "UNCHANGED"
    v = ug.verdict(_run(12), _run(0))
    assert v["verdict"] == "FIXED" and v["p"] < ug.FIXED_P
    assert "avoided" in ug.verdict(_run(12), _run(0, kernels=("k2",)))["why"]
    assert ug.verdict(_run(1), _run(0))["verdict"] == "INCONCLUSIVE"            # one failure in 20: not significant
    assert ug.verdict(_run(12), _run(0, log=False))["verdict"] == "INCONCLUSIVE"
    assert ug.verdict(_run(0, n=3), _run(0))["verdict"] == "INCONCLUSIVE"
    other = _run(0)
    other["conditions"] = {**other["conditions"], "gpu_name": "H100"}
    assert "gpu_name" in ug.verdict(_run(0), other)["why"]
    unknown = _run(0)
    del unknown["conditions"]["sms_visible"]
    assert ug.verdict(_run(0), unknown)["verdict"] == "INCONCLUSIVE"
    assert ug.verdict(_run(0), {"error": "boom"})["verdict"] == "INCONCLUSIVE"
    assert ug.exit_code(["PASSED", "FIXED"]) == 0
    assert ug.exit_code(["PASSED", "UNCHANGED"]) == 1
    assert ug.exit_code(["REGRESSED", "INCONCLUSIVE"]) == 2
    assert ug.exit_code([]) == 2


def test_fisher_tail():
    # 10 of 10 failures before, 0 of 10 after: P = 1 / C(20, 10)
    assert abs(ug.fisher_one_sided(10, 10, 0, 10) - 1 / 184756) < 1e-12
    assert ug.fisher_one_sided(0, 10, 0, 10) == 1.0


def test_tunableop_path():
    assert ug.tunableop_path("pin.csv", 0) == "pin0.csv"
    assert ug.tunableop_path("dir/p%d.csv", 3) == "dir/p3.csv"
    assert ug.tunableop_path("pin", 1) == "pin1"


def test_capture_run_compare_on_cpu(tmp_path, monkeypatch):
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "")
    pack = str(tmp_path / "gates")
    res = ug.capture((64, 128, 16), dtype="float32", bias=True, pack=pack, repeats=5, device="cpu")
    assert res["kind"] == "pin" and res["runs"] == 5 and res["runs_wrong"] == 0
    case = json.load(open(os.path.join(res["case"], "case.json")))
    assert case["schema"] == ug.CASE_SCHEMA and case["op"]["bias"] is True
    again = ug.capture((64, 128, 16), dtype="float32", bias=True, pack=pack, repeats=5, device="cpu")
    assert again["case"] == res["case"]                  # the same inputs: the first record is kept
    a = ug.run_pack(pack, repeats=5, device="cpu")
    b = ug.run_pack(pack, repeats=5, device="cpu")
    out = ug.compare(a, b)
    assert [v["verdict"] for v in out["cases"].values()] == ["PASSED"] and out["exit"] == 0


def test_judge_sees_wrong_and_unwritten():
    import torch
    x = torch.randn(4, 32, dtype=torch.float64)
    w = torch.randn(8, 32, dtype=torch.float64)
    ref, bound = ug.bound_and_ref(x, w, None, "float32")
    y = ref.float().clone()
    assert ug.judge(y, ref, bound)["wrong"] == 0
    y[1, 2] += 1.0
    y[3, 3] = float("nan")
    j = ug.judge(y, ref, bound)
    assert j["wrong"] == 2 and j["unwritten"] == 1


def test_cli_dispatch(monkeypatch):
    from sdcguard_b200 import cli
    called = {}
    monkeypatch.setattr(ug, "main", lambda argv: called.setdefault("ug", argv) and 0)
    cli.main(["gate", "compare", "a.json", "b.json"])
    assert called["ug"] == ["compare", "a.json", "b.json"]
    with pytest.raises(SystemExit):
        cli.main(["gate", "--help"])
