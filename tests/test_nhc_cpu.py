"""Node health check on the CPU with a stand-in check command: one line and exit 0 / 1 / 2, a hung check killed
at its deadline (whole process group), a FAIL that sticks until a clean check, and the cached mode's age rules."""
import json
import os
import sys
import time

from sdcguard_b200.tools import nhc


def _fake(kind):
    res = {"gemm_checks": 10, "gemm_wrong": 0, "copies_wrong": 0, "worst_z": 0.05}
    if kind == "fail":
        res.update(gemm_wrong=1, worst_z=1e9)
    code = {"ok": 0, "fail": 1, "noresult": 3}.get(kind, 0)
    body = (f"import json, time, sys; time.sleep({30 if kind == 'hang' else 0}); "
            f"print(json.dumps({res!r})) if {kind!r} != 'noresult' else None; sys.exit({code})")
    return lambda device, seconds: [sys.executable, "-c", body]


def test_ok_fail_sticky_and_clear(tmp_path):
    out = str(tmp_path / "nhc")
    line, code = nhc.run_nhc(["cuda:0", "cuda:1"], 1, out, command=_fake("ok"))
    assert code == 0 and line.startswith("OK: 2 GPUs")
    line, code = nhc.run_nhc(["cuda:0"], 1, out, command=_fake("fail"))
    assert code == 1 and line.startswith("FAIL")
    line, code = nhc.run_nhc(["cuda:0"], 1, out, command=_fake("noresult"))
    assert code == 1 and "a later check" in line                      # FAIL sticks over UNKNOWN
    line, code = nhc.run_nhc(["cuda:0"], 1, out, command=_fake("ok"))
    assert code == 0                                                   # a clean check clears it


def test_hung_check_is_killed_at_the_deadline(tmp_path):
    t0 = time.time()
    line, code = nhc.run_nhc(["cuda:0"], 1, str(tmp_path / "nhc"), command=_fake("hang"), limit=2.0)
    assert code == 2 and "did not finish" in line and time.time() - t0 < 20


def test_cached_mode(tmp_path):
    out = str(tmp_path / "nhc")
    assert nhc.cached(out, 24)[1] == 2
    nhc.write_status(out, "OK: fine", 0)
    assert nhc.cached(out, 24) == ("OK: fine", 0)
    st = json.load(open(os.path.join(out, "status.json")))
    st["time"] -= 48 * 3600
    json.dump(st, open(os.path.join(out, "status.json"), "w"))
    assert nhc.cached(out, 24)[1] == 2                                 # stale OK: unknown
    nhc.write_status(out, "FAIL: bad", 1)
    st = json.load(open(os.path.join(out, "status.json")))
    st["time"] -= 48 * 3600
    json.dump(st, open(os.path.join(out, "status.json"), "w"))
    assert nhc.cached(out, 24) == ("FAIL: bad", 1)                    # a FAIL is reported at any age


def test_chatty_checks_do_not_block_each_other(tmp_path):
    """Two checks that each write far more than a pipe buffer of log: both finish, neither is reported hung."""
    res = {"gemm_checks": 3, "gemm_wrong": 0, "copies_wrong": 0, "worst_z": 0.01}
    body = (f"import json, sys; sys.stderr.write('x' * (1 << 20)); sys.stderr.flush(); "
            f"print('y' * (1 << 19)); print(json.dumps({res!r}))")
    t0 = time.time()
    line, code = nhc.run_nhc(["cuda:0", "cuda:1"], 1, str(tmp_path / "nhc"),
                             command=lambda d, s: [sys.executable, "-c", body], limit=20.0)
    assert code == 0 and line.startswith("OK: 2 GPUs") and time.time() - t0 < 15
