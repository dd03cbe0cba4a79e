"""Recordings of this engine's prefill/decode transfer and the gate's verdicts on them (CPU: records only)."""
import contextlib
import io

from sdcguard_b200 import cli
from sdcguard_b200.coverage import observer as obs
from sdcguard_b200.serve import pd


def _gate(path):
    buf = io.StringIO()
    with contextlib.redirect_stdout(buf):
        rc = cli.main(["gate", str(path), "--require", "checksum"])
    return rc, buf.getvalue()


def _record(tmp_path, cases, reverify=()):
    rec = pd.Recorder()
    reqs = []
    for rid, n, local, bad in cases:
        sent = list(range(1, -(-n // 16) + 1))
        rec.transfer(rid, n, local, sent, bad)
        rec.cache("decode", rid, n, local, n - local, 8, "0" * 64)
        rec.cache("prefill", rid, n, 0, 0, 1, "0" * 64)
        if rid in reverify:
            rec.prefix_verified(rid, list(range(local // 16)), [])
        reqs.append((rid, list(range(n))))
    pd.write_recording(str(tmp_path), rec, reqs, {"engine_version": "test"})
    return rec


def test_full_transfer_passes(tmp_path):
    rec = _record(tmp_path, [("a", 166, 0, []), ("b", 40, 0, [])])
    v = rec.records[1]
    assert v["coverage"] == "complete" and v["native_result"] == "passed"
    rc, out = _gate(tmp_path)
    assert rc == 0 and "2 / 2 selected requests passed" in out


def test_cached_prefix_holds_unless_reverified(tmp_path):
    _record(tmp_path / "a", [("a", 166, 0, []), ("b", 166, 144, [])])
    rc, out = _gate(tmp_path / "a")
    assert rc == 2 and obs.CACHED_PREFIX_REASON in out and "1 / 2 selected requests passed" in out
    assert "transferred tokens checked: 22; decode cache reused unchecked: 144" in out
    _record(tmp_path / "b", [("a", 166, 0, []), ("b", 166, 144, [])], reverify={"b"})
    rc, out = _gate(tmp_path / "b")
    assert rc == 0 and "2 / 2 selected requests passed" in out


def test_mismatch_holds(tmp_path):
    rec = _record(tmp_path, [("a", 100, 0, [3])])
    assert rec.records[1]["native_result"] == "mismatch"
    rc, out = _gate(tmp_path)
    assert rc == 2 and "native_checksum_mismatch" in out


def test_tampered_recording_holds(tmp_path):
    _record(tmp_path, [("a", 100, 0, [])])
    p = tmp_path / "OBSERVER.json"
    p.write_bytes(p.read_bytes().replace(b'"complete"', b'"partial"', 1))
    rc, out = _gate(tmp_path)
    assert rc == 2 and "recording_file_digest_disagrees:OBSERVER.json" in out
