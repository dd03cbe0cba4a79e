"""The HTTP server on a B200 (tiny model, a subprocess) probed from outside: ready (with a probe request) says
PROTECTED, greedy outputs are isolated from their batch and decode agrees with prefill, throughput is measured; an
unchecked server reads NOT PROTECTED; qualify + decide accept an fp8 candidate against the bf16 baseline."""
import json
import os
import socket
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _cmd(port, extra=""):
    return f"{sys.executable} -m sdcguard_b200.serve.http --model tiny --port {port} --max-num-seqs 16 " \
           f"--max-model-len 512 {extra}"


def test_server_probes(tmp_path):
    from sdcguard_b200.tools import consistency, isolation, perf, ready
    from sdcguard_b200.tools.qualify import Server
    os.chdir(ROOT)
    port = _port()
    url = f"http://127.0.0.1:{port}"
    srv = Server(_cmd(port), url, str(tmp_path / "s.log"))
    try:
        r = ready.check(url, probe=True)
        assert r["verdict"] == "PROTECTED", r
        assert isolation.run(url, probes=2, primers=6)["verdict"] == "ISOLATED"
        c = consistency.run(url, probes=2)
        assert c["verdict"] == "CONSISTENT", c
        p = perf.run(url, clients=4, prompt=64, tokens=8, seconds=3)
        assert p["requests"] > 0 and p["errors"] == 0, p
    finally:
        srv.stop()
    port = _port()
    url = f"http://127.0.0.1:{port}"
    srv = Server(_cmd(port, "--unchecked"), url, str(tmp_path / "u.log"))
    try:
        assert ready.check(url, probe=True)["verdict"] == "NOT PROTECTED"
    finally:
        srv.stop()


def test_qualify_and_decide(tmp_path):
    from sdcguard_b200.tools import decide, qualify
    os.chdir(ROOT)
    p1, p2 = _port(), _port()
    out = str(tmp_path / "q")
    os.makedirs(out)
    base = qualify.run_one("baseline", _cmd(p1), f"http://127.0.0.1:{p1}", out, seconds=2, clients=4)
    cand = qualify.run_one("candidate", _cmd(p2, "--precision fp8"), f"http://127.0.0.1:{p2}", out, seconds=2,
                           clients=4)
    d = decide.decide(base, cand, {"waive": ["performance"]})
    assert d["sections"]["arithmetic"]["verdict"] == "NO FAULT OBSERVED", d
    assert d["decision"] == "ACCEPT", json.dumps(d["sections"])
    assert d["candidate_stack"]["precision"] == "fp8"
