"""The HTTP server's streaming completions, metrics and alert log on the CPU, with a fake engine in place of the GPU
one: the real server code, the real SSE client (`perf.stream_request`), `perf.measure`, `ready.check` and `decide`
reading the server's own metrics and alert log."""
import json
import socket
import threading
import time
from types import SimpleNamespace

import torch

from sdcguard_b200.serve import http as srv_http
from sdcguard_b200.serve.guard import ServeGuard
from sdcguard_b200.serve.settings import CheckSettings
from sdcguard_b200.tools import decide, perf, ready
from sdcguard_b200.utils.events import SDCEvent


class _State:
    def __init__(self):
        self.names = ["layers.0.qkv (ABFT GEMM)"]
        self.checks = 0

    def read(self, reset=True):
        rows = [{"name": self.names[0], "checks": self.checks, "unjudged": 0, "z": 0.1, "noise": 1.0, "flat": 0}]
        self.checks = 0
        return rows


class _Model:
    precision = "bf16"

    def __init__(self):
        self.settings = CheckSettings()
        self.state = _State()
        self.device = torch.device("cpu")
        self.embed = torch.zeros(8, 4)
        self.lm_head = torch.zeros(8, 4)
        self.final_ln = torch.ones(4)
        self.layers = []

    def check_coverage(self):
        return {"layers_checked": 3, "layers_unchecked": 0, "fp8_layers_checked": 0, "weights_checked_ratio": 1.0}


class _Engine:
    """Greedy 'model': token t+1 follows t. Tokens reach on_tokens one column at a time, as from the GPU tap."""

    def __init__(self):
        self.device = torch.device("cpu")
        self.checked = True
        self.max_num_seqs = 8
        self.cfg = SimpleNamespace(vocab=1000, name="fake")
        self.model = _Model()
        self.guard = ServeGuard(self.model)

    def generate(self, prompts, plens, new, on_tokens=None):
        N = prompts.shape[0]
        last = torch.tensor([int(prompts[i, plens[i] - 1]) for i in range(N)])
        out = torch.stack([(last + 1 + j) % 1000 for j in range(new)], 1)
        self.model.state.checks += N * new
        for col in range(new):
            if on_tokens is not None:
                on_tokens(list(range(N)), col, out[:, col].tolist())
            time.sleep(0.001)
        return out


def _serve():
    import uvicorn
    eng = _Engine()
    server = srv_http.Server(eng, "fake", batch_window_ms=2.0, max_prompt=512, digest="d0")
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    u = uvicorn.Server(uvicorn.Config(srv_http.make_app(server), host="127.0.0.1", port=port, log_level="error"))
    th = threading.Thread(target=u.run, daemon=True)
    th.start()
    url = f"http://127.0.0.1:{port}"
    for _ in range(200):
        try:
            if json.loads(srv_http_get(url + "/health")).get("ok"):
                break
        except OSError:
            time.sleep(0.05)
    return server, u, th, url


def srv_http_get(url):
    from sdcguard_b200.tools import _client
    return _client.get(url, 2.0)


def test_streaming_server_end_to_end(tmp_path):
    server, u, th, url = _serve()
    try:
        r = perf.stream_request(url, [5, 6, 7], 6)
        assert r["done"] and r["tokens"] == 6 and r["chunks"] == 6 and r["ttft_s"] > 0 and len(r["gaps_s"]) == 5
        from sdcguard_b200.tools import _client
        assert _client.complete(url, [5, 6, 7], 4) == [8, 9, 10, 11]
        m = perf.measure(url, perf.default_load(6, lo=4, hi=10), concurrency=3, max_tokens=5, rounds=2, warmup=1)
        assert m["complete"], m["why"]
        assert m["model"] == "fake" and m["median"]["ttft_p50_ms"] > 0 and m["median"]["itl_p50_ms"] > 0
        assert m["stack"]["weights_digest"] == "d0" and m["checks_on"] is True
        # ready: checks move with traffic
        rd = ready.check(url, probe=True)
        assert rd["verdict"] == "PROTECTED", rd
        # an alert in the server's log: the metrics count it and decide reads both
        alerts = tmp_path / "alerts.jsonl"
        server.eng.guard.log.path = str(alerts)
        server.eng.guard.log.add(SDCEvent(detector="checksum", step=1,
                                          detail={"layer": "layers.0.qkv", "recheck": {"verdict": "output_wrong"}}))
        text = _client.get(url + "/metrics")
        mm = _client.parse_metrics(text)
        assert mm["sdcguard_alerts_total"] == 1 and mm["sdcguard_confirmed_alerts_total"] == 1
        assert mm["sdcguard_layers_checked"] == 3 and mm["sdcguard_weights_checked_ratio"] == 1.0
        assert mm["sdcguard_longest_prompt_tokens"] >= 10
        assert ready.check(url)["verdict"] == "FAULT FOUND"
        d = decide.decide(None, quality={"verdict": "PASS", "mean_kl": 0, "top1_agreement": 1.0},
                          alerts=decide.read_alerts(str(alerts)), metrics=[text])
        assert d["decision"] == "REJECT" and d["arithmetic"]["verdict"] == "FAULT"
        # a bad prompt is a 400, not a stream
        try:
            perf.stream_request(url, [], 2)
            raise AssertionError("expected a failure")
        except perf.RequestFailed as e:
            assert "400" in str(e)
    finally:
        u.should_exit = True
        th.join(timeout=10)
        server.stop.set()
