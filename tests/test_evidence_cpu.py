"""Scoped assessment of a recorded P/D run (coverage gate + lifetime events) and the portable evidence bundle:
verdicts, offline verification, tampering and signatures."""
import json
import os

from sdcguard_b200.evidence import assessment, bundle
from sdcguard_b200.lifetime import adapter
from sdcguard_b200.serve import pd
from sdcguard_b200.tools import certify


def _recording(d, local=0, bad=()):
    rec = pd.Recorder()
    reqs = []
    for rid, n in (("a", 166), ("b", 40)):
        sent = list(range(1, -(-n // 16) + 1))
        rec.transfer(rid, n, local if rid == "a" else 0, sent, list(bad) if rid == "a" else [])
        rec.cache("decode", rid, n, local if rid == "a" else 0, n - (local if rid == "a" else 0), 8, "0" * 64)
        rec.cache("prefill", rid, n, 0, 0, 1, "0" * 64)
        reqs.append((rid, list(range(n))))
    pd.write_recording(str(d), rec, reqs, {"engine_version": "test"})


def _events(path, bad=False):
    s = adapter.EventSink(str(path))
    s.alloc("prefill", 0, "a")
    s.local_write("prefill", 0, "a")
    if bad:
        s.free("prefill", 0)
        s.alloc("prefill", 0, "z")
        s.local_write("prefill", 0, "z")
    s.alloc("decode", 1, "a")
    s.transfer("read", "pull", ("prefill", 0), ("decode", 1))
    s.consume("decode", 1, "a")
    s.close()
    return str(path)


def test_assessment_verdicts(tmp_path):
    _recording(tmp_path / "ok")
    assert assessment.assess(str(tmp_path / "ok"), _events(tmp_path / "ok.jsonl"))["verdict"] == "PASS"
    assert assessment.assess(str(tmp_path / "ok"))["verdict"] == "HOLD"           # no lifetime events
    r = assessment.assess(str(tmp_path / "ok"), _events(tmp_path / "bad.jsonl", bad=True))
    assert r["verdict"] == "FAIL" and r["lifetime"]["violations"][0]["rule"] == "R3"
    _recording(tmp_path / "cached", local=64)
    assert assessment.assess(str(tmp_path / "cached"), _events(tmp_path / "c.jsonl"))["verdict"] == "HOLD"
    _recording(tmp_path / "mism", bad=[3])
    assert assessment.assess(str(tmp_path / "mism"), _events(tmp_path / "m.jsonl"))["verdict"] == "FAIL"


def test_bundle_create_verify_tamper_sign(tmp_path):
    _recording(tmp_path / "rec")
    kp, pp = certify.keygen(str(tmp_path / "k"))
    out = str(tmp_path / "bundle")
    m = bundle.create(out, str(tmp_path / "rec"), _events(tmp_path / "ev.jsonl"), key=kp)
    assert m["assessment"]["verdict"] == "PASS" and "signature" in m
    assert bundle.verify(out, pp) == {"valid": True, "problems": [], "verdict": "PASS"}
    assert os.path.exists(bundle.report(out))
    os.remove(os.path.join(out, "report.html"))
    with open(os.path.join(out, "lifetime.jsonl"), "a") as f:
        f.write(json.dumps({"ev": "consume", "region": ["decode", 9], "gen": 0, "request": "x"}) + "\n")
    r = bundle.verify(out, pp)
    assert not r["valid"] and "changed: lifetime.jsonl" in r["problems"]
    assert any("re-assessment" in p for p in r["problems"])
