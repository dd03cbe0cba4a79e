"""The offline coverage gate, transfer-check and transfer-compare on the saved H100 recordings of the reference
(tests/data/checksum_owner_*): verdicts, exit codes and the full JSON output must equal the reference's own output
on the same inputs, byte for byte (digests in tests/data/golden_verdicts.json were taken from the reference CLI)."""
import contextlib
import hashlib
import io
import json
import shutil
import zipfile
from pathlib import Path

import pytest

from sdcguard_b200 import cli

DATA = Path(__file__).parent / "data"
GOLD = json.loads((DATA / "golden_verdicts.json").read_text())


def run(*argv):
    buf = io.StringIO()
    with contextlib.redirect_stdout(buf):
        rc = cli.main(list(argv))
    return rc, buf.getvalue()


def sha(s: str) -> str:
    return hashlib.sha256(s.encode()).hexdigest()


@pytest.mark.parametrize("rec", ["3a2ad847", "870c1aac", "9b42f5ab", "b340ee03"])
def test_gate_json_equals_reference(rec):
    rc, out = run("gate", str(DATA / f"checksum_owner_{rec}"), "--require", "checksum", "--json")
    assert rc == 2
    assert sha(out) == GOLD[f"gate_{rec}.json"]["sha256"]


def test_gate_text_reproduces_published_numbers():
    rc, out = run("gate", str(DATA / "checksum_owner_3a2ad847"), "--require", "checksum")
    assert rc == 2 and sha(out) == GOLD["gate_3a2ad847.txt"]["sha256"]
    assert "9 / 153 selected requests passed" in out
    assert "Prompt tokens: 1451; transferred tokens checked: 27; decode cache reused unchecked: 1424" in out


@pytest.mark.parametrize("rec,code", [("3a2ad847", 0), ("870c1aac", 2), ("9b42f5ab", 0), ("b340ee03", 0)])
def test_transfer_check_equals_reference(rec, code):
    rc, out = run("transfer-check", str(DATA / f"checksum_owner_{rec}"), "--json")
    assert rc == code
    assert sha(out) == GOLD[f"tc_{rec}.json"]["sha256"]


def test_transfer_compare_equals_reference():
    rc, out = run("transfer-compare", str(DATA / "checksum_owner_9b42f5ab"), str(DATA / "checksum_owner_b340ee03"),
                  "--json")
    assert rc == 2
    assert sha(out) == GOLD["cmp.json"]["sha256"]
    d = json.loads(out)
    assert d["summary"]["preserved"] == 153 and d["summary"]["regressed"] == 0


def _tampered(tmp_path, mutate):
    src = DATA / "checksum_owner_3a2ad847"
    dst = tmp_path / "rec"
    shutil.copytree(src, dst)
    zpath = dst / "ordinary-evidence.zip"
    with zipfile.ZipFile(zpath) as z:
        members = {i.filename: z.read(i) for i in z.infolist()}
    mutate(members)
    with zipfile.ZipFile(zpath, "w", zipfile.ZIP_DEFLATED) as z:
        for k, v in members.items():
            z.writestr(k, v)
    return dst


def test_tampered_native_result_holds(tmp_path):
    """A verification record whose stored verdict disagrees with its primitive observations holds the request."""
    def flip(members):
        name = "observer-on/decode/checksum-467.json"
        v = json.loads(members[name])
        for r in v["snapshot"]["records"]:
            if r["kind"] == "verification" and r["coverage"] == "complete":
                r["coverage"] = "partial"
                break
        members[name] = json.dumps(v).encode()
    rc, out = run("gate", str(_tampered(tmp_path, flip)), "--require", "checksum")
    assert rc == 2
    assert "0 / 153 selected requests passed" in out or "evidence" in out


def test_unreadable_archive_holds_with_reason(tmp_path):
    dst = tmp_path / "rec"
    shutil.copytree(DATA / "checksum_owner_3a2ad847", dst)
    (dst / "ordinary-evidence.zip").write_bytes(b"not a zip")
    rc, out = run("gate", str(dst), "--require", "checksum")
    assert rc == 2 and "evidence_unverifiable:unreadable owner archive" in out
