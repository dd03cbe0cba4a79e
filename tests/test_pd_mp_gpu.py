"""Multi-process prefill/decode on two GPUs (one prefill rank, one decode rank, torchrun): the decode rank pulls the
producer's KV pages over NVLink with the checksumming copy, its recording passes the gate when cached prefixes are
re-verified, its page lifetimes break no rule; a bit flipped in a producer page is caught (skipped with fewer than
2 GPUs)."""
import contextlib
import io
import json
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(out, extra=()):
    cmd = ["timeout", "-k", "30", "400", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(_port()), "-m",
           "sdcguard_b200.serve.pd_mp", "--prefill", "1", "--model", "tiny", "--groups", "2", "--per-group", "3",
           "--new-tokens", "4", "--out", str(out), *extra]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, env=env, timeout=500)
    if r.returncode != 0:
        i = r.stderr.find("Traceback")
        raise AssertionError(r.stderr[i:i + 4000] if i >= 0 else r.stderr[-3000:])
    return json.loads([x for x in r.stdout.splitlines() if x.startswith("{")][-1])


def _gate(p):
    from sdcguard_b200 import cli
    buf = io.StringIO()
    with contextlib.redirect_stdout(buf):
        rc = cli.main(["gate", str(p), "--require", "checksum"])
    return rc, buf.getvalue()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_pd_two_processes(tmp_path):
    r = _run(tmp_path / "ok", ["--verify-cached-prefix"])
    assert r["lifetime_violations"] == 0 and r["ranks_with_mismatch"] == 0 and r["tokens_per_s"] > 0, r
    rc, out = _gate(tmp_path / "ok" / "decode0")
    assert rc == 0 and "6 / 6 selected requests passed" in out, out
    from sdcguard_b200.evidence import assessment
    a = assessment.assess(str(tmp_path / "ok" / "decode0"), str(tmp_path / "ok" / "decode0" / "lifetime.jsonl"))
    assert a["verdict"] == "PASS", a
    r = _run(tmp_path / "bad", ["--verify-cached-prefix", "--corrupt-page", "0"])
    assert r["ranks_with_mismatch"] == 1, r
    rc, out = _gate(tmp_path / "bad" / "decode0")
    assert rc == 2 and "native_checksum_mismatch" in out, out
