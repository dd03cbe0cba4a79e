"""The protection metrics a serving worker publishes (Prometheus text), one rendering for this package's HTTP server
and for the vLLM plugin's per-worker exporter, so `sdcguard ready`, `decide` and `qualify` read either the same way.

    text = render(coverage, check_coverage, counters, worker, stack, settings, z_alarm, scan=None)
    exporter = Exporter(port, lambda: text_now())     # GET /metrics on 0.0.0.0:port from a daemon thread

Names: sdcguard_protected, _checks_total, _alarms_total, _unjudged_total, _ops_total / _ops_checked,
_sampled_ops_total / _run, _alarm_line, _worst_clean_z, _polls_total, _requests_total, _prompt_tokens_total,
_generated_tokens_total, _longest_prompt_tokens, _layers_checked / _unchecked, _weights_checked_ratio,
_fp8_layers_checked, _fp8_calls_judged_total, _fp8_findings_total, _alerts_total, _confirmed_alerts_total, the weight
scan's series when it runs, and the info series sdcguard_worker_info{gpu, uuid, pid, started, device},
sdcguard_stack_info{model, precision, checked, torch, cuda, weights_digest, version} and
sdcguard_protection_info{share, offset, norms, rope, attn, act, spot, z, weight_scan}.

Reference: the metrics the reference's plugin exports for `sdcguard ready` (src/sdcguard/ready.py:1-40,
SDCGUARD_METRICS_PORT in src/sdcguard/vllm_plugin.py).
"""
from __future__ import annotations

import threading
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer
from typing import Callable, Optional


def _labels(d: dict) -> str:
    return ",".join(f'{k}="{str(v).lower() if isinstance(v, bool) else v}"' for k, v in d.items())


def render(cov: dict, check_cov: dict, counters: dict, worker: dict, stack: dict, settings: dict, z_alarm: float,
           scan: Optional[dict] = None, protected: bool = True) -> str:
    c = {"polls": 0, "requests": 0, "prompt_tokens": 0, "generated_tokens": 0, "longest_prompt": 0, **counters}
    cc = {"layers_checked": 0, "layers_unchecked": 0, "fp8_layers_checked": 0, "weights_checked_ratio": 0.0,
          **(check_cov or {})}
    lines = [
        "# TYPE sdcguard_protected gauge", f"sdcguard_protected {1 if protected else 0}",
        "# TYPE sdcguard_checks_total counter", f"sdcguard_checks_total {cov.get('checks', 0)}",
        f"sdcguard_alarms_total {cov.get('alarms', 0)}", f"sdcguard_unjudged_total {cov.get('unjudged', 0)}",
        f"sdcguard_ops_total {cov.get('ops', 0)}", f"sdcguard_ops_checked {cov.get('ops_checked', 0)}",
        f"sdcguard_sampled_ops_total {cov.get('sampled_ops', 0)}",
        f"sdcguard_sampled_ops_run {cov.get('sampled_ops_run', 0)}",
        f"sdcguard_alarm_line {z_alarm}", f"sdcguard_worst_clean_z {cov.get('worst_clean_z', 0.0)}",
        f"sdcguard_polls_total {c['polls']}", f"sdcguard_requests_total {c['requests']}",
        f"sdcguard_prompt_tokens_total {c['prompt_tokens']}",
        f"sdcguard_generated_tokens_total {c['generated_tokens']}",
        f"sdcguard_longest_prompt_tokens {c['longest_prompt']}",
        f"sdcguard_layers_checked {cc['layers_checked']}", f"sdcguard_layers_unchecked {cc['layers_unchecked']}",
        f"sdcguard_weights_checked_ratio {cc['weights_checked_ratio']:.6f}",
        f"sdcguard_fp8_layers_checked {cc['fp8_layers_checked']}",
        f"sdcguard_fp8_calls_judged_total {cov.get('fp8_calls_judged', 0)}",
        f"sdcguard_fp8_findings_total {cov.get('fp8_findings', 0)}",
        f"sdcguard_alerts_total {cov.get('alerts', 0)}",
        f"sdcguard_confirmed_alerts_total {cov.get('confirmed_alerts', 0)}",
        f"sdcguard_worker_info{{{_labels(worker)}}} 1",
        f"sdcguard_stack_info{{{_labels(stack)}}} 1",
        f"sdcguard_protection_info{{{_labels(settings)}}} 1",
    ]
    if scan is not None:
        lines += [f"sdcguard_weight_scan_entries {scan['entries']}",
                  f"sdcguard_weight_scan_passes_total {scan['passes']}",
                  f"sdcguard_weight_scan_never_compared {scan['never_compared']}",
                  f"sdcguard_weight_scan_changed {scan['changed']}",
                  f"sdcguard_weight_repairs_total {scan['repairs']}",
                  f"sdcguard_weight_scan_left_out {scan['left_out']}"]
        if scan.get("oldest_age_seconds") is not None:
            lines.append(f"sdcguard_weight_scan_oldest_age_seconds {scan['oldest_age_seconds']:.3f}")
    return "\n".join(lines) + "\n"


def settings_labels(settings, z_alarm: float, weight_scan: bool) -> dict:
    """The protection_info labels of a `serve.settings.CheckSettings` (or {} without one)."""
    prot = dict(settings.describe()) if settings is not None else {}
    prot.pop("notes", None)
    prot["z"] = prot.pop("z_alarm", z_alarm)
    prot["weight_scan"] = bool(weight_scan)
    return prot


class Exporter:
    """GET /metrics from a daemon thread (the text comes from `text()` at each request); close() stops it."""

    def __init__(self, port: int, text: Callable[[], str], host: str = "0.0.0.0"):
        class Handler(BaseHTTPRequestHandler):
            def do_GET(self):  # noqa: N802  (http.server's method name)
                if self.path.split("?")[0] not in ("/metrics", "/"):
                    self.send_error(404)
                    return
                try:
                    body = text().encode()
                except Exception as e:  # noqa: BLE001  (a scrape that fails is a 500, never a dead worker)
                    self.send_error(500, str(e)[:200])
                    return
                self.send_response(200)
                self.send_header("Content-Type", "text/plain; version=0.0.4")
                self.send_header("Content-Length", str(len(body)))
                self.end_headers()
                self.wfile.write(body)

            def log_message(self, *a):
                pass

        self.httpd = ThreadingHTTPServer((host, port), Handler)
        self.port = self.httpd.server_address[1]
        self.thread = threading.Thread(target=self.httpd.serve_forever, daemon=True)
        self.thread.start()

    def close(self) -> None:
        self.httpd.shutdown()
        self.httpd.server_close()
