"""Host-side tools: cuBLASLt log inventory, coverage and diff; the known-issue matcher."""
from sdcguard_b200.tools import kernels, known_issues

K66 = ("algoId=66 tile=MATMUL_TILE_64x16 stages=MATMUL_STAGES_64xAUTO customOption=1 "
       "clusterShape=CLUSTER_SHAPE_4x1x1")
SPLIT = "algoId=66 tile=MATMUL_TILE_64x32 stages=MATMUL_STAGES_8x3 reductionScheme=REDUCTION_SCHEME_COMPUTE_TYPE numSplitsK=8"


def _line(m, n, k, algo=K66, t="R_16BF", transa="OP_T", fn="cublasLtMatmul"):
    a_rows, a_cols = (k, m) if transa == "OP_T" else (m, k)
    return (f"[2026-12-01 10:00:00][cublasLt][7][Trace][{fn}] A=0X1 Adesc=[type={t} rows={a_rows} cols={a_cols} "
            f"ld={a_rows}] B=0X2 Bdesc=[type={t} rows={k} cols={n} ld={k}] C=0X3 Cdesc=[type={t} rows={m} cols={n} "
            f"ld={m}] D=0X3 Ddesc=[type={t} rows={m} cols={n} ld={m}] computeDesc=[computeType=COMPUTE_32F "
            f"scaleType=R_32F transa={transa}] algo=[{algo}] workSpaceSizeInBytes=0")


def test_parse_line_and_keys():
    c = kernels.parse_line(_line(1000, 16, 2048))
    assert (c["m"], c["n"], c["k"]) == (1000, 16, 2048) and c["types"] == ["bf16"] * 4
    assert c["algo"]["clusterShape"] == "4x1x1" and c["algo"]["tile"] == "64x16"
    assert "algoId=66 tile=64x16 stages=64xAUTO customOption=1 clusterShape=4x1x1" in kernels.kernel_key(c)
    p = kernels.parse_line(_line(64, 8, 32, transa="OP_N"))
    assert (p["m"], p["n"], p["k"]) == (64, 8, 32)
    assert kernels.parse_line("[cublasLt][7][Api][cublasLtMatmul] A=0X1") is None
    assert kernels.parse_line("unrelated") is None


def test_inventory_coverage_diff_and_flags():
    work = kernels.inventory([_line(1536, 16, 8960)] * 3 + [_line(256, 16, 1536, algo=SPLIT),
                                                            "[cublasLt][7][Trace][cublasLtMatmul] A=0X1 broken", "x"])
    assert work["calls"] == 4 and work["unreadable_lines"] == 1 and len(work["kernels"]) == 2
    shares = sorted(e["work_share"] for e in work["kernels"].values())
    assert abs(sum(shares) - 1) < 1e-6
    flagged = [e["flags"] for e in work["kernels"].values()]
    assert any("6862950" in f[0] for f in flagged if f) and any(any("6580689" in x for x in f) for f in flagged)
    test = kernels.inventory([_line(1536, 16, 8960), _line(64, 64, 64, t="R_32F")])
    cov = kernels.coverage(work, [test])
    assert cov["kernels"] == 2 and cov["kernels_exercised"] == 1 and len(cov["not_exercised"]) == 1
    assert cov["work_exercised"] == cov["work_exercised_same_shape"] > 0.5
    d = kernels.diff(work, test)
    assert len(d["only_before"]) == 1 and len(d["only_after"]) == 1 and d["both"] == 1


def test_known_issue_verdicts():
    rows = {r["id"]: r["verdict"] for r in known_issues.match({"cublas": (12, 9, 1), "cc": "10.0",
                                                               "mps_percentage": None})}
    assert rows["6862950"] == "not affected"           # Hopper only
    assert rows["5807900"] == "may apply"              # fixed on the 12.9 branch at 12.9.2
    assert known_issues.match({"cublas": (12, 9, 2), "cc": "10.0"})[3]["verdict"] == "not affected"
    hop = {r["id"]: r["verdict"] for r in known_issues.match({"cublas": (12, 8, 0), "cc": "9.0",
                                                              "mps_percentage": 50.0})}
    assert hop["6862950"] == "applies"
    hop = {r["id"]: r["verdict"] for r in known_issues.match({"cublas": (12, 8, 0), "cc": "9.0"})}
    assert hop["6862950"] == "not active"


def test_gate_model_kl_and_verdict_lines():
    import math

    import torch

    from sdcguard_b200.tools import gate_model
    v = torch.log(torch.tensor([0.5, 0.3, 0.2]))
    i = torch.tensor([4, 7, 9])
    assert abs(gate_model.compare_position(v, i, v, i)) < 1e-12
    # candidate moved mass from token 4 to 7 and lists a new token 11
    cv = torch.log(torch.tensor([0.4, 0.4, 0.2]))
    kl = gate_model.compare_position(v, i, cv, torch.tensor([4, 7, 11]))
    assert kl > 0.01
    base = {"mean_kl": 1e-4, "top1_agreement": 1.0, "worst_prompt_kl": 1e-3, "positions": 1000}
    assert gate_model.verdict(base)["verdict"] == "PASS"
    assert gate_model.verdict({**base, "mean_kl": 5e-3})["verdict"] == "WARN"
    assert gate_model.verdict({**base, "top1_agreement": 0.9})["verdict"] == "FAIL"
    noisy = {"mean_kl": 2e-3, "top1_agreement": 0.985, "worst_prompt_kl": 0.04}
    assert gate_model.verdict({**base, "mean_kl": 5e-3, "top1_agreement": 0.984}, noisy)["verdict"] == "PASS"
    assert math.isclose(gate_model.verdict(base, noisy)["lines"]["pass_kl"], 6e-3)


def _case(wrong=True):
    import torch

    from sdcguard_b200.tools import casefile
    g = torch.Generator().manual_seed(0)
    x = torch.randn(4, 256, generator=g).bfloat16()
    w = (torch.randn(256, 256, generator=g) * 0.05).bfloat16()
    y = (x.float() @ w.float().t()).bfloat16()
    if wrong:
        y[2, 130] = y[2, 130] * 4 + 1
    c = casefile.capture(x, w, y, 2, 1)
    c["stack"] = {"torch": "t", "cuda": "c", "gpu_name": "B200", "gpu_uuid": "GPU-A", "cublas": None, "cc": None}
    return c


def test_casefile_explanations():
    from sdcguard_b200.tools import casefile
    c = _case()
    rc = casefile.recheck(c)
    assert rc["output_wrong"] and rc["first_bad_column"] == 130
    h = casefile.sha256(c)
    st = dict(c["stack"])
    here = {"case_sha256": h, "gpu_uuid": "GPU-A", "stack": st, "runs": 20, "reproduced": 0}
    peer = {"case_sha256": h, "gpu_uuid": "GPU-B", "stack": {**st, "gpu_uuid": "GPU-B"}, "runs": 20, "reproduced": 0}
    r = casefile.casefile(c, [here, peer])
    assert r["outcome"] == "most consistent with: transient fault on the incident GPU", r
    r = casefile.casefile(c, [{**here, "reproduced": 5}, peer])
    assert r["outcome"] == "most consistent with: persistent defect of the incident GPU", r
    r = casefile.casefile(c, [{**here, "reproduced": 5}, {**peer, "reproduced": 3}])
    assert r["outcome"] == "most consistent with: software or library defect", r
    r = casefile.casefile(c, [{**here, "case_sha256": "other"}])
    assert r["outcome"] == "INCONCLUSIVE" and r["replays"]["ignored_other_case"] == 1 and r["next_steps"]
    ok = _case(wrong=False)
    assert casefile.casefile(ok, [])["outcome"] == "most consistent with: false alarm of the check"


def test_investigate_classification():
    from sdcguard_b200.tools.investigate import classify
    ok = {"checked_kernel_wrong": 0, "library_wrong": 0, "alarms": 0}
    ours = {"checked_kernel_wrong": 3, "library_wrong": 0, "alarms": 3}
    both = {"checked_kernel_wrong": 3, "library_wrong": 2, "alarms": 3}
    assert classify([ok, ok], []) == "NOT REPRODUCED"
    assert classify([ours, ok], []) == "DEVICE"
    assert classify([ours, ours], []) == "SOFTWARE PATH"
    assert classify([both, both], []) == "NOT ONE GPU"
    assert classify([ours], []) == "INCONCLUSIVE"
    assert classify([ok], [{"error": "x"}]) == "INCONCLUSIVE"


def test_replay_command_refuses_what_it_cannot_run(tmp_path):
    from sdcguard_b200 import cli
    assert cli.main(["replay", str(tmp_path / "missing.pt")]) == 2
    assert cli.main(["replay", str(tmp_path / "missing.pt"), "--times", "0"]) == 2


def test_kernel_test_verdicts(tmp_path):
    """`kernels test` bookkeeping with a fake replay worker: PASSED when the same kernel ran and every run was right,
    OTHER KERNEL when another kernel ran, WRONG on a wrong run, NOT RUN for types it does not replay."""
    inv = kernels.inventory([_line(1536, 16, 8960), _line(256, 16, 1536, algo=SPLIT), _line(128, 8, 64),
                             _line(64, 64, 64, t="R_32F")])
    seen = {}

    def runner(todo, log_dir):
        seen["todo"] = todo
        res = []
        for t in todo:
            res.append({"runs": 3, "runs_wrong": 1 if t["m"] == 128 else 0, "runs_unwritten": 0})
        # here the 1536-row shape runs the inventory's kernel, the 256-row one another
        lines = [_line(1536, 16, 8960), _line(256, 16, 1536), _line(128, 8, 64)]
        return {"results": res, "gpu": "fake"}, lines

    r = kernels.test_calls(inv, repeats=3, log_dir=str(tmp_path), runner=runner)
    v = {c["call"].split(" | ")[1].split(" batch")[0]: c["verdict"] for c in r["calls"]}
    assert v["m=1536 n=16 k=8960"] == "PASSED"
    assert v["m=256 n=16 k=1536"] == "OTHER KERNEL"
    assert v["m=128 n=8 k=64"] == "WRONG"
    assert v["m=64 n=64 k=64"] == "NOT RUN"
    assert r["counts"] == {"PASSED": 1, "WRONG": 1, "OTHER KERNEL": 1, "NOT RUN": 1}
    assert len(seen["todo"]) == 3 and all(t["dtype"] == "bf16" and t["transa"] == "OP_T" for t in seen["todo"])
    # the decision reads the report: one judged call on the workload's kernel makes it a source, WRONG a fault
    from sdcguard_b200.tools import decide
    w = decide.kernel_test_witness(r)
    assert w.tested == 2 and w.faults and not w.unresolved


def test_kernel_test_output_judgement():
    import torch
    a = torch.randn(8, 32, dtype=torch.float64)
    b = torch.randn(32, 4, dtype=torch.float64)
    ref = a @ b
    y = ref.to(torch.bfloat16)
    assert kernels.judge_output(y, ref, a.abs(), b.abs(), 32, "bf16") == {"wrong": 0, "unwritten": 0}
    bad = y.clone()
    bad[1, 2] += 4.0
    assert kernels.judge_output(bad, ref, a.abs(), b.abs(), 32, "bf16")["wrong"] == 1
    bad[0, 0] = float("nan")
    assert kernels.judge_output(bad, ref, a.abs(), b.abs(), 32, "bf16")["unwritten"] == 1
