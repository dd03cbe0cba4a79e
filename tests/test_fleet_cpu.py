"""Certificates (Ed25519 sign / verify, tampering, evidence hashes, expiry), the fleet view (quarantine list, RMA zip)
and the results board (validation, aggregation, fingerprint reference), on synthetic reports."""
import datetime as dt
import json
import os

from sdcguard_b200.tools import board, certify, fleet
from sdcguard_b200.tools.check import SCHEMA, card_digest


def _screen(verdict="PASS", uuid="GPU-1", evidence=None):
    rounds = [{"round": 0, "tokens": 100, "alarms": 0, "mismatched_tokens": 0}]
    if evidence:
        rounds.append({"round": 1, "tokens": 100, "alarms": 1, "mismatched_tokens": 0, "evidence": evidence})
    return {"gpu": "NVIDIA B200", "size": "tiny", "seed": 0, "tokens": 200, "checks": 1234, "verdict": verdict,
            "failed_rounds": [1] if evidence else [], "worst_clean_z": 0.1, "rounds": rounds,
            "telemetry_before": {"uuid": uuid, "serial": "S1", "pci.bus_id": "0000:1B:00.0", "name": "NVIDIA B200"}}


def test_certificate_sign_verify_and_tamper(tmp_path):
    kp, pp = certify.keygen(str(tmp_path / "fleet"))
    d = tmp_path / "gpu1"
    d.mkdir()
    ev = d / "evidence_r1.pt"
    ev.write_bytes(b"evidence bytes")
    cert = certify.sign(certify.make(_screen("FAIL", evidence=str(ev)), base_dir=str(d)), kp)
    p = d / "certificate.json"
    p.write_text(json.dumps(cert))
    r = certify.verify(str(p), pp)
    assert r["valid"] and r["verdict"] == "FAIL", r
    ev.write_bytes(b"changed")
    assert "evidence changed: evidence_r1.pt" in certify.verify(str(p), pp)["problems"]
    ev.write_bytes(b"evidence bytes")
    cert["result"]["verdict"] = "PASS"                 # tampered after signing
    p.write_text(json.dumps(cert))
    assert "bad signature" in certify.verify(str(p), pp)["problems"]
    late = dt.datetime.now(dt.timezone.utc) + dt.timedelta(days=60)
    good = certify.sign(certify.make(_screen()), kp)
    p.write_text(json.dumps(good))
    assert certify.verify(str(p), pp, now=late)["problems"] == ["expired"]


def test_fleet_quarantines_failures(tmp_path):
    for name, verdict, uuid in (("a", "PASS", "GPU-A"), ("b", "FAIL", "GPU-B")):
        d = tmp_path / "root" / name
        d.mkdir(parents=True)
        (d / "screen.json").write_text(json.dumps(_screen(verdict, uuid)))
    d = tmp_path / "root" / "c"
    d.mkdir()
    (d / "screen_ops.json").write_text(json.dumps({"verdict": "FAIL", "telemetry_before": {"uuid": "GPU-C"},
                                                   "tests": {"fma_fp32": {"verdict": "FAIL"}}}))
    rows = fleet.collect([str(tmp_path / "root")])
    st = {r["gpu"]: r["status"] for r in rows}
    assert st == {"GPU-A": "ok", "GPU-B": "quarantine", "GPU-C": "quarantine"}
    s = fleet.write(rows, str(tmp_path / "out"))
    assert s["quarantined"] == 2 and len(s["rma_zips"]) == 2
    assert sorted(open(tmp_path / "out" / "quarantine.txt").read().split()) == ["GPU-B", "GPU-C"]
    assert "GPU-B" in open(tmp_path / "out" / "fleet.html").read()


def _card(result="PASS", gid="h1", fp="f1", wrong=0, minutes=2.0):
    c = {"schema": SCHEMA, "result": result, "gpu": {"name": "NVIDIA B200", "id_hash": gid},
         "versions": {}, "minutes": minutes,
         "speed": {"checked_tflops": 1300.0, "cublas_tflops": 1500.0, "d2d_gbs": 6400.0},
         "checked": {"gemm_checks": 100, "copies_verified": 1000, "wrong": wrong, "worst_z": 0.1},
         "fingerprint": {"key": "NVIDIA B200|8192|0|12.8", "output": fp}, "provider": "p"}
    c["digest"] = card_digest(c)
    return c


def test_board_validates_and_aggregates(tmp_path):
    d = tmp_path / "cards"
    d.mkdir()
    cards = [_card(gid="h1"), _card(gid="h2"), _card(gid="h3", fp="f2", result="FAIL", wrong=3),
             _card(gid="h4", minutes=0.2)]
    bad = _card(gid="h5")
    bad["speed"]["checked_tflops"] = 2e9
    for i, c in enumerate(cards + [bad]):
        (d / f"c{i}.json").write_text(json.dumps(c))
    s = board.build([str(d)], str(tmp_path / "out"))
    assert s["accepted"] == 3 and s["rejected"] == 2 and s["FAIL"] == 1
    ref = json.load(open(tmp_path / "out" / "reference.json"))["fingerprints"]["NVIDIA B200|8192|0|12.8"]
    assert ref == {"f1": 2, "f2": 1}
    agg = board.aggregate(board.load([str(d)])[0])
    assert agg["models"]["NVIDIA B200"]["fingerprint_agreement"] == [2, 3]
    assert os.path.exists(tmp_path / "out" / "index.html")


def test_reference_command_names(tmp_path, capsys):
    """`sdcguard keygen`, `verify` and `report`, the reference's names for certify keygen / verify and fleet
    collect, give the same results."""
    from sdcguard_b200 import cli
    assert cli.main(["keygen", "--out", str(tmp_path / "k")]) == 0
    kp, pp = str(tmp_path / "k") + ".key", str(tmp_path / "k") + ".pub"
    keys = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    kp, pp = keys.get("private", kp), keys.get("public", pp)
    d = tmp_path / "root" / "node1"
    d.mkdir(parents=True)
    good = certify.sign(certify.make(_screen()), kp)
    (d / "certificate.json").write_text(json.dumps(good))
    assert cli.main(["verify", str(d / "certificate.json"), "--pubkey", pp]) == 0
    bad = dict(good, result=dict(good["result"], verdict="FAIL"))
    (tmp_path / "bad.json").write_text(json.dumps(bad))
    assert cli.main(["verify", str(d / "certificate.json"), str(tmp_path / "bad.json"), "--pubkey", pp]) == 1
    capsys.readouterr()
    rc = cli.main(["report", str(tmp_path / "root"), "--out", str(tmp_path / "rep"), "--pubkey", pp])
    assert rc in (0, 1) and (tmp_path / "rep" / "fleet.html").exists()
    assert cli.COMMANDS["demo"] is not None
