"""Offline evidence packets (native-checks over the saved owner recordings): capture writes inputs, report and a
manifest; verify recomputes the report and refuses a packet whose files were changed."""
import json
import os
import shutil

import pytest

from sdcguard_b200.coverage import packets

DATA = os.path.join(os.path.dirname(__file__), "data")


@pytest.mark.parametrize("rec", ["checksum_owner_3a2ad847", "checksum_owner_b340ee03"])
def test_native_checks_packet_round_trip(tmp_path, rec, capsys):
    from sdcguard_b200.coverage.gate import inspect
    owner = os.path.join(DATA, rec)
    out = str(tmp_path / "packet")
    rc = packets.native_main(["capture", "--owner-result", owner, "--out", out, "--require", "checksum", "--json"])
    rep = json.loads(capsys.readouterr().out)
    gate = inspect(owner, ["checksum"])
    assert rep["release"] == gate["decision"] and rc == (0 if gate["decision"] == "PASS" else 2)
    assert rep["gate"] == json.loads(json.dumps(gate))
    man = json.load(open(os.path.join(out, "manifest.json")))
    assert "report.json" in man["files"] and any(n.startswith("inputs/owner/") for n in man["files"])
    assert packets.native_main(["verify", out]) == rc
    # a changed input is refused
    victim = next(n for n in man["files"] if n.startswith("inputs/owner/") and n.endswith(".json"))
    with open(os.path.join(out, victim), "ab") as f:
        f.write(b" ")
    assert packets.native_main(["verify", out]) == 2
    assert "inconclusive" in capsys.readouterr().out
    with pytest.raises(packets.ev.EvidenceError):
        packets.verify(out, "native-checks")
    # a packet is written once
    shutil.rmtree(out)
    packets.native_main(["capture", "--owner-result", owner, "--out", out])
    assert packets.native_main(["capture", "--owner-result", owner, "--out", out]) == 2


def test_observer_and_client_reject_wrong_inputs(tmp_path, capsys):
    bad = tmp_path / "s.json"
    bad.write_text(json.dumps({"schema": "something else"}))
    assert packets.observer_main(["inspect", str(bad)]) == 2
    assert "inconclusive" in capsys.readouterr().out
    assert packets.client_main(["inspect", "--plan", str(bad), "--inventory", str(bad), "--captures", str(bad)]) == 2
