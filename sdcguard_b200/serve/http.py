"""HTTP front end of the checked serving engine: an OpenAI-style completions endpoint, Prometheus metrics that say
from outside whether (and how much) the math is being checked, and a stack-identity record.

    python -m sdcguard_b200.serve.http --model tiny --port 8000 [--unchecked] [--precision fp8]

Endpoints
  POST /v1/completions   {"prompt": [token ids] or "text", "max_tokens": n, "stream": false}; greedy decoding. Text
                         prompts use a byte-level mapping (byte value mod vocab): the models are random-init shapes,
                         not trained. Returns {"choices": [{"token_ids": [...], "text": "..."}], "usage": {...}}.
                         With "stream": true the answer is server-sent events: one `data: {choices: [{text,
                         token_ids}]}` per token as the GPU produces it, then `data: {choices: [], usage: {...}}` and
                         `data: [DONE]` (what a client measures time to first token and inter-token latency from).
  GET  /metrics          sdcguard_protected, sdcguard_checks_total, sdcguard_alarms_total, sdcguard_unjudged_total,
                         sdcguard_ops_total / _checked, sdcguard_alarm_line, sdcguard_worst_clean_z,
                         sdcguard_polls_total (check results read back), sdcguard_requests_total,
                         sdcguard_prompt_tokens_total, sdcguard_generated_tokens_total,
                         sdcguard_longest_prompt_tokens; what is checked:
                         sdcguard_layers_checked / _unchecked, sdcguard_weights_checked_ratio,
                         sdcguard_fp8_layers_checked, sdcguard_fp8_calls_judged_total, sdcguard_fp8_findings_total;
                         alerts: sdcguard_alerts_total, sdcguard_confirmed_alerts_total (an alert with its own evidence
                         of a wrong result); the weight scan (--weight-scan-mb): sdcguard_weight_scan_entries,
                         _passes_total, _never_compared, _changed, _repairs_total, _left_out, _oldest_age_seconds;
                         sdcguard_worker_info{gpu, uuid, pid, started}, sdcguard_stack_info{model, precision, checked,
                         torch, cuda, weights_digest, version} and sdcguard_protection_info{share, offset, norms, rope,
                         attn, act, spot, z, weight_scan} (the check settings a qualification ran with).
  POST /v1/score         {"prompt": [token ids], "top_k": k}: teacher-forced top-k log-probabilities of every position
                         (one prefill): {"top_logprobs": [[...]], "top_ids": [[...]]}, position p predicting token p + 1.
  GET  /health, GET /v1/models, GET /sdcguard/status (coverage report and events as JSON).

Requests are batched: a worker thread takes the first waiting request and every other one that arrives within the
batch window (up to max_num_seqs), runs one generate() for all of them, and truncates each to its max_tokens. The
check state is polled after every batch, so the counters move with the traffic.

Reference: the vLLM plugin's metrics exporter and stack record that `sdcguard ready` reads
(src/sdcguard/ready.py:1-40, src/sdcguard/vllm_plugin.py); here the engine is this library's own.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import queue
import threading
import time
from typing import Optional

import torch

from ..models.decoder import CONFIGS
from ..numerics import abft


class Request:
    def __init__(self, ids: list[int], max_tokens: int, score_topk: int = 0, stream: bool = False):
        self.ids, self.max_tokens = ids, max_tokens
        self.score_topk = score_topk          # > 0: a teacher-forced scoring request instead of a generation
        self.done = threading.Event()
        self.out: Optional[list[int]] = None
        self.error: Optional[str] = None
        # streaming: token ids as they are produced, then None (or an error string) at the end
        self.tokens: Optional["queue.Queue"] = queue.Queue() if stream else None
        self.sent = 0


def model_weights(model) -> list:
    """(name, tensor) of every weight of a checked decoder: embedding, per-layer projections and norms, LM head
    (entries a layer does not have are skipped)."""
    out = [("embed", model.embed)]
    for i, lw in enumerate(model.layers):
        for name in ("ln1", "ln2", "qkv", "o", "gate_up", "down", "q_norm", "k_norm"):
            out.append((f"layers.{i}.{name}", getattr(lw, name, None)))
    if model.lm_head is not model.embed:
        out.append(("lm_head", model.lm_head))
    out.append(("final_norm", getattr(model, "final_ln", None)))
    return [(n, t) for n, t in out if t is not None]


class Server:
    def __init__(self, engine, model_name: str, batch_window_ms: float = 5.0, max_prompt: int = 2048,
                 weight_scan_mb: float = 0.0, alerts_path: Optional[str] = None, digest: Optional[str] = None):
        self.eng = engine
        self.model_name = model_name
        self.window = batch_window_ms / 1000.0
        self.max_prompt = max_prompt
        self.q: "queue.Queue[Request]" = queue.Queue()
        self.counters = {"requests": 0, "prompt_tokens": 0, "generated_tokens": 0, "polls": 0, "batches": 0,
                         "longest_prompt": 0}
        self.events: list = []
        self.started = time.time()
        self.lock = threading.Lock()
        self.stop = threading.Event()
        if alerts_path:
            self.eng.guard.log.path = alerts_path
        self.scan = None
        if weight_scan_mb > 0:
            from .weights import WeightScan
            self.scan = WeightScan(model_weights(self.eng.model), log=self.eng.guard.log)
            self.eng.guard.attach_weight_scan(self.scan, weight_scan_mb)
        self.digest = digest or self._weights_digest()
        self.thread = threading.Thread(target=self._worker, daemon=True)
        self.thread.start()

    def _weights_digest(self) -> str:
        from ..ops.fingerprint import fingerprint
        ws = [t for _, t in model_weights(self.eng.model) if t is not None]
        fp = fingerprint(ws)
        return hashlib.sha256(fp.cpu().numpy().tobytes()).hexdigest()[:16]

    def tokens(self, prompt) -> list[int]:
        V = self.eng.cfg.vocab
        ids = [int(t) % V for t in prompt] if isinstance(prompt, list) else [b % V for b in str(prompt).encode()]
        if not ids or len(ids) > self.max_prompt:
            raise ValueError(f"prompt must have 1 to {self.max_prompt} tokens")
        return ids

    def submit(self, ids: list[int], max_tokens: int, timeout: float = 600.0) -> list[int]:
        r = Request(ids, max(1, int(max_tokens)))
        self.q.put(r)
        if not r.done.wait(timeout):
            raise TimeoutError("request timed out")
        if r.error:
            raise RuntimeError(r.error)
        return r.out

    def submit_stream(self, ids: list[int], max_tokens: int) -> Request:
        """Queue a streaming request; its .tokens queue yields ids as they are produced, then None (or an error
        string)."""
        r = Request(ids, max(1, int(max_tokens)), stream=True)
        self.q.put(r)
        return r

    @staticmethod
    def _emit(batch: list, rows, col: int, ids: list) -> None:
        for r_i, tok in zip(rows, ids):
            r = batch[r_i]
            if r.tokens is not None and col < r.max_tokens:
                r.tokens.put(int(tok))
                r.sent += 1

    def score(self, ids: list[int], topk: int, timeout: float = 600.0) -> dict:
        """Teacher-forced top-k log-probabilities of every position of `ids` (one prefill, checks included)."""
        r = Request(ids, 0, score_topk=max(1, min(int(topk), 20)))
        self.q.put(r)
        if not r.done.wait(timeout):
            raise TimeoutError("request timed out")
        if r.error:
            raise RuntimeError(r.error)
        return r.out

    def _run_score(self, r: Request) -> None:
        try:
            (v, i), = self.eng.score([r.ids], r.score_topk)
            ev = self.eng.guard.poll()
            with self.lock:
                self.events.extend(ev)
                self.counters["polls"] += 1
                self.counters["requests"] += 1
                self.counters["prompt_tokens"] += len(r.ids)
                self.counters["longest_prompt"] = max(self.counters["longest_prompt"], len(r.ids))
            r.out = {"top_logprobs": v.tolist(), "top_ids": i.tolist()}
        except Exception as e:  # noqa: BLE001  (returned to the request)
            r.error = f"{type(e).__name__}: {e}"
        r.done.set()

    def _worker(self) -> None:
        if torch.device(self.eng.device).type == "cuda":
            torch.cuda.set_device(self.eng.device)
        while not self.stop.is_set():
            try:
                first = self.q.get(timeout=0.1)
            except queue.Empty:
                continue
            if first.score_topk:
                self._run_score(first)
                continue
            batch = [first]
            t_end = time.time() + self.window
            while len(batch) < self.eng.max_num_seqs:
                left = t_end - time.time()
                if left <= 0:
                    break
                try:
                    nxt = self.q.get(timeout=left)
                except queue.Empty:
                    break
                if nxt.score_topk:            # scoring runs on its own, after this batch
                    self._run_score(nxt)
                    continue
                batch.append(nxt)
            try:
                L = max(len(r.ids) for r in batch)
                prompts = torch.zeros(len(batch), L, dtype=torch.long)
                for i, r in enumerate(batch):
                    prompts[i, : len(r.ids)] = torch.tensor(r.ids)
                new = max(r.max_tokens for r in batch)
                tap = None
                if any(r.tokens is not None for r in batch):
                    tap = lambda rows, col, ids, b=batch: self._emit(b, rows, col, ids)  # noqa: E731
                pin = prompts.pin_memory() if torch.cuda.is_available() else prompts
                out = self.eng.generate(pin, [len(r.ids) for r in batch], new, on_tokens=tap)
                ev = self.eng.guard.poll()
                with self.lock:
                    self.events.extend(ev)
                    self.counters["polls"] += 1
                    self.counters["batches"] += 1
                    self.counters["requests"] += len(batch)
                    self.counters["prompt_tokens"] += sum(len(r.ids) for r in batch)
                    self.counters["generated_tokens"] += sum(r.max_tokens for r in batch)
                    self.counters["longest_prompt"] = max([self.counters["longest_prompt"]]
                                                          + [len(r.ids) for r in batch])
                for i, r in enumerate(batch):
                    r.out = out[i, : r.max_tokens].tolist()
                    if r.tokens is not None:
                        for tok in r.out[r.sent:]:        # anything the tap did not deliver
                            r.tokens.put(int(tok))
                        r.tokens.put(None)
                    r.done.set()
            except Exception as e:  # noqa: BLE001  (returned to every request of the batch)
                for r in batch:
                    r.error = f"{type(e).__name__}: {e}"
                    if r.tokens is not None:
                        r.tokens.put(r.error)
                    r.done.set()

    def metrics(self) -> str:
        from .. import __version__
        from .metrics import render, settings_labels
        g = self.eng.guard
        dev = torch.device(self.eng.device)
        if dev.type == "cuda":
            props = torch.cuda.get_device_properties(dev)
            gpu, uuid = props.name, str(getattr(props, "uuid", ""))
        else:
            gpu, uuid = "cpu", ""
        stack = {"model": self.model_name, "precision": getattr(self.eng.model, "precision", "bf16"),
                 "checked": str(self.eng.checked).lower(), "torch": torch.__version__, "cuda": torch.version.cuda,
                 "weights_digest": self.digest, "version": __version__}
        worker = {"gpu": gpu, "uuid": uuid, "pid": os.getpid(), "started": int(self.started), "device": dev}
        cc = self.eng.model.check_coverage() if self.eng.checked else None
        return render(g.coverage_report(), cc, self.counters, worker, stack,
                      settings_labels(getattr(self.eng.model, "settings", None), g.z_alarm, self.scan is not None),
                      g.z_alarm, self.scan.stats() if self.scan is not None else None, protected=self.eng.checked)

    def status(self) -> dict:
        with self.lock:
            ev = [{"detector": e.detector, "detail": e.detail, "time": e.time} for e in self.events[-100:]]
        return {"coverage": self.eng.guard.coverage_report(), "events": ev, "counters": dict(self.counters),
                "alarm_line": abft.Z_ALARM}


def sse(server: Server, r: Request, timeout: float = 600.0):
    """Server-sent events of a streaming request: a chunk per token, the usage chunk, [DONE]; an error event (and no
    [DONE]) when generation failed."""
    n = 0
    t_end = time.time() + timeout
    while True:
        try:
            tok = r.tokens.get(timeout=1.0)
        except queue.Empty:
            if not server.thread.is_alive():
                tok = "the server's batch worker stopped"
            elif time.time() > t_end:
                tok = "request timed out"
            else:
                continue
        if tok is None:
            break
        if isinstance(tok, str):
            yield "event: error\n" + "data: " + json.dumps({"error": tok}) + "\n\n"
            return
        n += 1
        yield "data: " + json.dumps({"object": "text_completion", "model": server.model_name,
                                     "choices": [{"index": 0, "text": f" {tok}", "token_ids": [tok],
                                                  "finish_reason": None}]}) + "\n\n"
    usage = {"prompt_tokens": len(r.ids), "completion_tokens": n, "total_tokens": len(r.ids) + n}
    yield "data: " + json.dumps({"object": "text_completion", "model": server.model_name,
                                 "choices": [{"index": 0, "text": "", "finish_reason": "length"}]}) + "\n\n"
    yield "data: " + json.dumps({"choices": [], "usage": usage}) + "\n\n"
    yield "data: [DONE]\n\n"


def make_app(server: Server):
    from fastapi import FastAPI, HTTPException
    from fastapi.responses import PlainTextResponse, StreamingResponse
    app = FastAPI()

    @app.post("/v1/completions")
    def completions(body: dict):
        if body.get("stream"):
            try:
                ids = server.tokens(body.get("prompt", ""))
            except ValueError as e:
                raise HTTPException(status_code=400, detail=str(e)) from e
            r = server.submit_stream(ids, int(body.get("max_tokens", 16)))
            return StreamingResponse(sse(server, r), media_type="text/event-stream")
        try:
            ids = server.tokens(body.get("prompt", ""))
            out = server.submit(ids, int(body.get("max_tokens", 16)))
        except ValueError as e:
            raise HTTPException(status_code=400, detail=str(e)) from e
        except (RuntimeError, TimeoutError) as e:
            raise HTTPException(status_code=500, detail=str(e)) from e
        return {"object": "text_completion", "model": server.model_name,
                "choices": [{"index": 0, "token_ids": out, "text": " ".join(map(str, out)), "finish_reason": "length"}],
                "usage": {"prompt_tokens": len(ids), "completion_tokens": len(out),
                          "total_tokens": len(ids) + len(out)}}

    @app.post("/v1/score")
    def score(body: dict):
        """{"prompt": token ids, "top_k": k} -> per position p the top-k log-probabilities of token p + 1."""
        try:
            ids = server.tokens(body.get("prompt", ""))
            return server.score(ids, int(body.get("top_k", 5)))
        except ValueError as e:
            raise HTTPException(status_code=400, detail=str(e)) from e
        except (RuntimeError, TimeoutError) as e:
            raise HTTPException(status_code=500, detail=str(e)) from e

    @app.get("/metrics", response_class=PlainTextResponse)
    def metrics():
        return server.metrics()

    @app.get("/health")
    def health():
        return {"ok": server.thread.is_alive()}

    @app.get("/v1/models")
    def models():
        return {"data": [{"id": server.model_name, "object": "model"}]}

    @app.get("/sdcguard/status")
    def status():
        return server.status()

    return app


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m sdcguard_b200.serve.http")
    ap.add_argument("--model", default="tiny", help=f"one of {sorted(CONFIGS)}")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--device", default="cuda:0")
    ap.add_argument("--unchecked", action="store_true")
    ap.add_argument("--precision", default="bf16", choices=["bf16", "fp8"])
    ap.add_argument("--max-num-seqs", type=int, default=32)
    ap.add_argument("--max-model-len", type=int, default=2048)
    ap.add_argument("--batch-window-ms", type=float, default=5.0)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--weight-scan-mb", type=float, default=float(os.environ.get("SDCGUARD_WEIGHT_SCAN_MB", "0")),
                    help="fingerprint this many MB of weights after every batch and compare with the load "
                         "(0: off; SDCGUARD_WEIGHT_SCAN_MB)")
    ap.add_argument("--alerts", default=os.environ.get("SDCGUARD_LOG"),
                    help="append every alert as a JSON line to this file (SDCGUARD_LOG)")
    a = ap.parse_args(argv)
    import uvicorn
    from .engine import LLMEngine
    cfg = CONFIGS[a.model]
    eng = LLMEngine(cfg, device=a.device, checked=not a.unchecked, max_num_seqs=a.max_num_seqs,
                    max_prefill_tokens=a.max_num_seqs * a.max_model_len // 2, max_model_len=a.max_model_len,
                    kv_fraction=0.3, seed=a.seed, precision=a.precision)
    srv = Server(eng, cfg.name, a.batch_window_ms, max_prompt=a.max_model_len // 2,
                 weight_scan_mb=a.weight_scan_mb, alerts_path=a.alerts)
    uvicorn.run(make_app(srv), host=a.host, port=a.port, log_level="warning")
    srv.stop.set()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
