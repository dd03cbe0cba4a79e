"""HTTP front end of the checked serving engine: an OpenAI-style completions endpoint, Prometheus metrics that say
from outside whether (and how much) the math is being checked, and a stack-identity record.

    python -m sdcguard_b200.serve.http --model tiny --port 8000 [--unchecked] [--precision fp8]

Endpoints
  POST /v1/completions   {"prompt": [token ids] or "text", "max_tokens": n}; greedy decoding. Text prompts use a
                         byte-level mapping (byte value mod vocab): the models are random-init shapes, not trained.
                         Returns {"choices": [{"token_ids": [...], "text": "..."}], "usage": {...}}.
  GET  /metrics          sdcguard_protected, sdcguard_checks_total, sdcguard_alarms_total, sdcguard_unjudged_total,
                         sdcguard_ops_total / _checked, sdcguard_alarm_line, sdcguard_worst_clean_z,
                         sdcguard_polls_total (check results read back), sdcguard_requests_total,
                         sdcguard_prompt_tokens_total, sdcguard_generated_tokens_total, sdcguard_worker_info{gpu, uuid,
                         pid, started} and sdcguard_stack_info{model, precision, checked, torch, cuda, weights_digest}.
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
import os
import queue
import threading
import time
from typing import Optional

import torch

from ..models.decoder import CONFIGS
from ..numerics import abft


class Request:
    def __init__(self, ids: list[int], max_tokens: int, score_topk: int = 0):
        self.ids, self.max_tokens = ids, max_tokens
        self.score_topk = score_topk          # > 0: a teacher-forced scoring request instead of a generation
        self.done = threading.Event()
        self.out: Optional[list[int]] = None
        self.error: Optional[str] = None


class Server:
    def __init__(self, engine, model_name: str, batch_window_ms: float = 5.0, max_prompt: int = 2048):
        self.eng = engine
        self.model_name = model_name
        self.window = batch_window_ms / 1000.0
        self.max_prompt = max_prompt
        self.q: "queue.Queue[Request]" = queue.Queue()
        self.counters = {"requests": 0, "prompt_tokens": 0, "generated_tokens": 0, "polls": 0, "batches": 0}
        self.events: list = []
        self.started = time.time()
        self.lock = threading.Lock()
        self.stop = threading.Event()
        self.digest = self._weights_digest()
        self.thread = threading.Thread(target=self._worker, daemon=True)
        self.thread.start()

    def _weights_digest(self) -> str:
        from ..ops.fingerprint import fingerprint
        m = self.eng.model
        ws = [m.embed] + [t for lw in m.layers for t in (lw.qkv, lw.o, lw.gate_up, lw.down)]
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
            r.out = {"top_logprobs": v.tolist(), "top_ids": i.tolist()}
        except Exception as e:  # noqa: BLE001  (returned to the request)
            r.error = f"{type(e).__name__}: {e}"
        r.done.set()

    def _worker(self) -> None:
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
                out = self.eng.generate(prompts.pin_memory(), [len(r.ids) for r in batch], new)
                ev = self.eng.guard.poll()
                with self.lock:
                    self.events.extend(ev)
                    self.counters["polls"] += 1
                    self.counters["batches"] += 1
                    self.counters["requests"] += len(batch)
                    self.counters["prompt_tokens"] += sum(len(r.ids) for r in batch)
                    self.counters["generated_tokens"] += sum(r.max_tokens for r in batch)
                for i, r in enumerate(batch):
                    r.out = out[i, : r.max_tokens].tolist()
                    r.done.set()
            except Exception as e:  # noqa: BLE001  (returned to every request of the batch)
                for r in batch:
                    r.error = f"{type(e).__name__}: {e}"
                    r.done.set()

    def metrics(self) -> str:
        g = self.eng.guard
        cov = g.coverage_report()
        dev = self.eng.device
        props = torch.cuda.get_device_properties(dev)
        uuid = str(getattr(props, "uuid", ""))
        c = self.counters
        stack = {"model": self.model_name, "precision": getattr(self.eng.model, "precision", "bf16"),
                 "checked": str(self.eng.checked).lower(), "torch": torch.__version__, "cuda": torch.version.cuda,
                 "weights_digest": self.digest}
        lab = ",".join(f'{k}="{v}"' for k, v in stack.items())
        lines = [
            "# TYPE sdcguard_protected gauge", f"sdcguard_protected {1 if self.eng.checked else 0}",
            "# TYPE sdcguard_checks_total counter", f"sdcguard_checks_total {cov['checks']}",
            f"sdcguard_alarms_total {cov['alarms']}", f"sdcguard_unjudged_total {cov['unjudged']}",
            f"sdcguard_ops_total {cov['ops']}", f"sdcguard_ops_checked {cov['ops_checked']}",
            f"sdcguard_sampled_ops_total {cov['sampled_ops']}", f"sdcguard_sampled_ops_run {cov['sampled_ops_run']}",
            f"sdcguard_alarm_line {g.z_alarm}", f"sdcguard_worst_clean_z {cov['worst_clean_z']}",
            f"sdcguard_polls_total {c['polls']}", f"sdcguard_requests_total {c['requests']}",
            f"sdcguard_prompt_tokens_total {c['prompt_tokens']}",
            f"sdcguard_generated_tokens_total {c['generated_tokens']}",
            f'sdcguard_worker_info{{gpu="{props.name}",uuid="{uuid}",pid="{os.getpid()}",'
            f'started="{int(self.started)}",device="{dev}"}} 1',
            f"sdcguard_stack_info{{{lab}}} 1",
        ]
        return "\n".join(lines) + "\n"

    def status(self) -> dict:
        with self.lock:
            ev = [{"detector": e.detector, "detail": e.detail, "time": e.time} for e in self.events[-100:]]
        return {"coverage": self.eng.guard.coverage_report(), "events": ev, "counters": dict(self.counters),
                "alarm_line": abft.Z_ALARM}


def make_app(server: Server):
    from fastapi import FastAPI, HTTPException
    from fastapi.responses import PlainTextResponse
    app = FastAPI()

    @app.post("/v1/completions")
    def completions(body: dict):
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
    a = ap.parse_args(argv)
    import uvicorn
    from .engine import LLMEngine
    cfg = CONFIGS[a.model]
    eng = LLMEngine(cfg, device=a.device, checked=not a.unchecked, max_num_seqs=a.max_num_seqs,
                    max_prefill_tokens=a.max_num_seqs * a.max_model_len // 2, max_model_len=a.max_model_len,
                    kv_fraction=0.3, seed=a.seed, precision=a.precision)
    srv = Server(eng, cfg.name, a.batch_window_ms, max_prompt=a.max_model_len // 2)
    uvicorn.run(make_app(srv), host=a.host, port=a.port, log_level="warning")
    srv.stop.set()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
