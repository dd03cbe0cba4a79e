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
