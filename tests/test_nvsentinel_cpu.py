"""NVSentinel health events: wire encoding read back by an independent protobuf reader, events from a check result
and from a job's alert log, and a batch delivered to a gRPC server on a unix socket (with the bearer token), with
the publisher's rate limit."""
import json
import os
import time

import pytest

from sdcguard_b200.utils import nvsentinel as nv


def _read(buf: bytes) -> list:
    """(field, wire type, value) triples of one message level (varint -> int, length-delimited -> bytes)."""
    out, i = [], 0
    while i < len(buf):
        key, i = _varint(buf, i)
        num, wt = key >> 3, key & 7
        if wt == 0:
            v, i = _varint(buf, i)
        elif wt == 2:
            n, i = _varint(buf, i)
            v, i = buf[i:i + n], i + n
        else:
            raise AssertionError(f"wire type {wt}")
        out.append((num, wt, v))
    return out


def _varint(b, i):
    shift = n = 0
    while True:
        c = b[i]
        i += 1
        n |= (c & 0x7F) << shift
        shift += 7
        if c < 0x80:
            return n, i


def test_encoding_fields():
    ev = nv.HealthEvent(message="m", healthy=False, fatal=True, action="RUN_FIELDDIAG", codes=["A", "B"],
                        entities=[("PCI", "0000:1b:00.0"), ("GPU_UUID", "GPU-1")], metadata={"z": 1, "a": "x"},
                        when=1700000000.25, node="n1", strategy="EXECUTE_REMEDIATION")
    f = _read(ev.encode())
    nums = [x[0] for x in f]
    assert nums == sorted(nums)                          # field-number order
    d = {}
    for num, _, v in f:
        d.setdefault(num, []).append(v)
    assert d[1] == [1] and d[2] == [b"sdcguard"] and d[4] == [b"GpuComputeCorrectness"]
    assert d[5] == [1] and 6 not in d                    # fatal, unhealthy (false is not written)
    assert d[8] == [6] and d[9] == [b"A", b"B"] and d[16] == [1] and d[13] == [b"n1"]
    ents = [dict((n, v) for n, _, v in _read(e)) for e in d[10]]
    assert ents[1] == {1: b"GPU_UUID", 2: b"GPU-1"}
    meta = [dict((n, v) for n, _, v in _read(e)) for e in d[11]]
    assert [m[1] for m in meta] == [b"a", b"z"]          # map entries sorted by key
    ts = dict((n, v) for n, _, v in _read(d[12][0]))
    assert ts == {1: 1700000000, 2: 250000000}
    batch = _read(nv.encode_batch([ev, ev]))
    assert batch[0] == (1, 0, 1) and [x[0] for x in batch[1:]] == [2, 2]
    assert nv.Wire.varint(-1) == b"\xff" * 9 + b"\x01"


def test_events_from_check_and_alerts():
    assert nv.pci_entity("00000000:1B:00.0") == "0000:1b:00.0"
    ev, why = nv.from_check({"result": "FAIL", "gpu_uuid": "GPU-9", "pci_bus_id": "00000000:1B:00.0",
                             "device": "NVIDIA B200", "gemm_wrong": 1}, node="n", remediate=True)
    assert ev.fatal and ev.action == "RUN_FIELDDIAG" and ev.strategy == "EXECUTE_REMEDIATION"
    assert ("GPU_UUID", "GPU-9") in ev.entities and ("PCI", "0000:1b:00.0") in ev.entities
    ok, _ = nv.from_check({"result": "PASS", "gpu_uuid": "GPU-9"})
    assert ok.healthy and not ok.fatal and ok.strategy == "STORE_AND_ANALYSE"
    assert nv.from_check({"result": "INCOMPLETE", "gpu_uuid": "GPU-9"})[0] is None
    assert nv.from_check({"result": "PASS"})[0] is None
    host = "hostA"
    alerts = [{"detector": "checksum", "time": 10.0 + i, "detail": {"z": 9.0 + i, "layer": "L1.qkv"},
               "identity": {"gpu_uuid": "GPU-1", "host": host, "gpu_name": "B200"}} for i in range(3)]
    alerts.append({"detector": "checksum", "detail": {}, "identity": {"gpu_uuid": "GPU-2", "host": "other"}})
    alerts.append({"detector": "replay", "detail": {}, "identity": {}})
    evs, skipped = nv.from_alerts(alerts, node="n", host=host)
    assert len(evs) == 1 and len(skipped) == 2
    e = evs[0]
    assert not e.healthy and not e.fatal and e.codes == ["SDCGUARD_CHECKSUM"]
    assert e.metadata["alerts"] == "3" and e.metadata["worst_z"] == "11.0" and e.when == 12.0


def test_send_to_grpc_server_and_publisher(tmp_path):
    grpc = pytest.importorskip("grpc")
    from concurrent import futures
    got = []

    def handler(req, ctx):
        got.append((req, dict(ctx.invocation_metadata())))
        return b""

    sock = str(tmp_path / "nvs.sock")
    server = grpc.server(futures.ThreadPoolExecutor(max_workers=2))
    rpc = grpc.unary_unary_rpc_method_handler(handler, request_deserializer=None, response_serializer=None)
    server.add_generic_rpc_handlers((grpc.method_handlers_generic_handler(
        "datamodels.PlatformConnector", {"HealthEventOccurredV1": rpc}),))
    server.add_insecure_port(f"unix://{sock}")
    server.start()
    try:
        tok = tmp_path / "token"
        tok.write_text("secret\n")
        ev, _ = nv.from_check({"result": "PASS", "gpu_uuid": "GPU-3"}, node="n")
        nv.send([ev], socket_path=sock, token_file=str(tok), timeout=5)
        assert len(got) == 1 and got[0][0] == nv.encode_batch([ev])
        assert got[0][1].get("authorization") == "Bearer secret"
        pub = nv.Publisher(socket_path=sock, token_file=str(tok), node="n", min_interval=3600)
        from sdcguard_b200.utils.events import SDCEvent
        ident = {"gpu_uuid": "GPU-4", "host": os.uname().nodename}
        for _ in range(3):
            pub(SDCEvent(detector="spot", step=1, detail={"z": 50.0}, identity=ident))
        pub.flush()
        assert pub.sent == 1 and pub.skipped == 2 and pub.failed == 0
        assert len(got) == 2
    finally:
        server.stop(None)
    with pytest.raises(nv.SendError):
        nv.send([ev], socket_path=str(tmp_path / "missing.sock"))


def test_cli_dry_run(tmp_path, capsys):
    p = tmp_path / "check.json"
    p.write_text(json.dumps({"result": "FAIL", "gpu_uuid": "GPU-7", "device": "B200"}))
    assert nv.main([str(p), "--dry-run", "--node", "n"]) == 0
    out = json.loads(capsys.readouterr().out)
    assert out["events"][0]["isHealthy"] is False and out["events"][0]["nodeName"] == "n"
