"""CPU: alert delivery (webhook to a local HTTP endpoint, handler chain), Prometheus metrics, stack identity and
the clock-sample summary used for the bench's clock record."""
import http.server
import json
import threading
import time

from sdcguard_b200.utils import alerts, gpuinfo, stack
from sdcguard_b200.utils.events import SDCEvent


def test_webhook_posts_slack_payload_and_chain_survives_a_failing_handler():
    got = []

    class H(http.server.BaseHTTPRequestHandler):
        def do_POST(self):
            n = int(self.headers["Content-Length"])
            got.append(json.loads(self.rfile.read(n)))
            self.send_response(200)
            self.end_headers()

        def log_message(self, *a):
            pass

    srv = http.server.HTTPServer(("127.0.0.1", 0), H)
    threading.Thread(target=srv.serve_forever, daemon=True).start()
    hook = alerts.Webhook(f"http://127.0.0.1:{srv.server_address[1]}/x", kind="slack")
    seen = []

    def boom(ev):
        raise RuntimeError("handler failure")
    run = alerts.chain(boom, hook, seen.append)
    ev = SDCEvent(detector="checksum", step=7, detail={"layer": "layers.3.o", "row": 5, "block": 2},
                  identity={"host": "h", "gpu_uuid": "GPU-x"})
    run(ev)
    for _ in range(100):
        if got:
            break
        time.sleep(0.05)
    hook.close()
    srv.shutdown()
    assert seen == [ev]
    assert got and "layers.3.o" in got[0]["text"] and "step 7" in got[0]["text"]


def test_metrics_and_stack_identity():
    m = alerts.Metrics()
    m.on_event(SDCEvent(detector="replay", step=1))
    m.observe_coverage({"checks": 10, "unjudged": 1, "worst_clean_z": 0.5})
    s1 = {"model": "a", "torch": "2", "checked": True}
    m.publish_stack(s1)
    t = m.text().decode()
    assert 'sdcguard_alarms_total{detector="replay"} 1.0' in t and "sdcguard_worst_clean_z 0.5" in t
    s2 = dict(s1, model="b")
    assert stack.field_differences(s1, s2) == {"model": {"a": "a", "b": "b"}}
    assert stack.fingerprint(s1) != stack.fingerprint(s2)
    base = {"model": "m", "model_config": "c", "weights_digest": "w", "precision": "bf16", "library_build": "l",
            "gpu": "B200", "device": "cuda:0"}
    assert stack.compare(base, dict(base, device="cuda:3"))["same"] is True          # per-worker field
    r = stack.compare(base, dict(base, precision="fp8"))
    assert r["same"] is False and "precision" in r["why"]
    no_digest = {k: v for k, v in base.items() if k != "weights_digest"}
    assert stack.compare(base, no_digest)["same"] is None
    assert stack.compare(no_digest, no_digest)["same"] is None
    assert stack.compare(None, base)["same"] is None
    assert stack.shared(base) == stack.shared(dict(base, device="cuda:1", pid="9"))
    page = 'x 1\nsdcguard_stack_info{model="m",gpu="B200"} 1.0\n'
    assert stack.from_metrics(page) == {"model": "m", "gpu": "B200"}


def test_clock_sample_summary():
    lines = ["0, 1965, 1965, 900.1, 0x0, Not Active, Not Active, Not Active, Not Active",
             "0, 1900, 1965, 990.0, 0x4, Not Active, Not Active, Not Active, Active",
             "garbage"]
    s = gpuinfo.parse_samples(lines)
    assert s["samples"] == 2 and s["sm_max_mhz"] == 1965 and s["reasons"] == ["sw_power_cap"]
    assert gpuinfo.datasheet("NVIDIA B200")["bf16"] == 2250.0
