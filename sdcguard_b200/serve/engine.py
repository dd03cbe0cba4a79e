"""Single-GPU serving engine for the checked decoder: paged KV cache with 16-token pages, prefill batches
bounded by a token budget, then batched decode replayed from a CUDA graph, with the generated tokens kept on
the device until the end of the call (no host synchronisation per step).

    eng = LLMEngine(QWEN3_0_6B, checked=True)
    out = eng.generate(prompts, prompt_lens, max_new_tokens=128)   # pinned int64 host tensors in, host out
    report = eng.guard.poll()                                       # check results (see serve/guard.py)

Checks in every step (checked=True): ABFT on every GEMM row; exact replay of a rotating 1/`sample_every`
sample of rows for the norms, the q/k norm + RoPE + KV-cache write, attention and the activation.

Reference: the serving stack is vLLM in the reference (src/sdcguard/vllm_plugin.py, `GPUModelRunner.execute_model`
patch :2430-2501 with mark_step/poll); here the engine is this package's own, with the same hook points
(`serve.plugin`).
"""
from __future__ import annotations

import queue
import threading
import time
from dataclasses import dataclass
from typing import Callable, Optional, Sequence

import torch

from ..utils.trace import nvtx_range
from ..models.decoder import CheckedDecoder, DecoderConfig, StepMeta
from ..ops import attention
from .guard import ServeGuard

PAGE = 16


class BlockAllocator:
    """Free list of KV pages (page 0 is reserved as a never-read zero page)."""

    def __init__(self, num_blocks: int):
        self.num_blocks = num_blocks
        self.free = list(range(num_blocks - 1, 0, -1))

    def alloc(self, n: int) -> list[int]:
        if n > len(self.free):
            raise RuntimeError(f"KV cache full: need {n} pages, {len(self.free)} free")
        out = [self.free.pop() for _ in range(n)]
        return out

    def release(self, pages: Sequence[int]) -> None:
        self.free.extend(reversed(list(pages)))


def kv_bytes_per_page(cfg: DecoderConfig, nkv: int) -> int:
    return cfg.layers * 2 * nkv * PAGE * cfg.head_dim * 2


class TokenTap:
    """Hands each generated token column to a host callback as soon as the GPU has written it, without making the
    launching thread wait: after a column is produced, the engine queues a copy of it into pinned memory and an
    event on the stream; a tap thread waits for the events in order and calls on_tokens(rows, column, ids).

    Only generate() calls that pass on_tokens pay for this (one small copy and an event per step)."""

    def __init__(self, device: torch.device, n: int, max_new: int, on_tokens: Callable):
        self.host = torch.empty(max_new, n, dtype=torch.long, pin_memory=True)
        self.device = device
        self.on_tokens = on_tokens
        self.q: "queue.Queue" = queue.Queue()
        self.error: Optional[BaseException] = None
        self.thread = threading.Thread(target=self._run, daemon=True)
        self.thread.start()

    def push(self, rows: Sequence[int], col: int, src: torch.Tensor) -> None:
        """src: the column's tokens for `rows` (a contiguous range), on the device."""
        r0 = rows[0]
        self.host[col, r0:r0 + len(rows)].copy_(src, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        self.q.put((list(rows), col, ev))

    def _run(self) -> None:
        while True:
            item = self.q.get()
            if item is None:
                return
            rows, col, ev = item
            try:
                ev.synchronize()
                r0 = rows[0]
                self.on_tokens(rows, col, self.host[col, r0:r0 + len(rows)].tolist())
            except BaseException as e:  # noqa: BLE001  (kept and raised by close())
                self.error = self.error or e

    def close(self) -> None:
        self.q.put(None)
        self.thread.join()
        if self.error is not None:
            raise self.error


class LLMEngine:
    def __init__(self, cfg: DecoderConfig, device="cuda", checked: bool = True, num_blocks: Optional[int] = None,
                 max_prefill_tokens: int = 16384, max_num_seqs: int = 256, sample_every: int = 64,
                 cuda_graph: bool = True, seed: int = 0, kv_fraction: float = 0.6, model: Optional[CheckedDecoder] = None,
                 max_model_len: int = 4096, precision: str = "bf16", cache: Optional[torch.Tensor] = None):
        self.cfg = cfg
        self.device = torch.device(device)
        # a checked engine trusts this library's kernels on this device only after they reproduced their
        # references on clean and corrupted cases (once per device and process)
        self.verification = None
        if checked and self.device.type == "cuda":
            from ..ops import gemm, verify
            self.verification = verify.verified(self.device)
            gemm.enable_capture(self.device)      # the first alarm's evidence is kept on the device
        self.model = model or CheckedDecoder(cfg, self.device, checked=checked, seed=seed, precision=precision)
        self.checked = self.model.checked
        self.max_prefill_tokens = max_prefill_tokens
        self.max_num_seqs = max_num_seqs
        self.sample_every = sample_every
        self.cuda_graph = cuda_graph
        if cache is not None:          # caller-owned KV memory (e.g. a symmetric buffer peers read from)
            want = (cfg.layers, cache.shape[1], 2, self.model.nkv, PAGE, cfg.head_dim)
            if tuple(cache.shape) != want or cache.dtype != torch.bfloat16:
                raise ValueError(f"cache must be bf16 {want}, got {tuple(cache.shape)} {cache.dtype}")
            num_blocks = cache.shape[1]
            self.cache = cache
        else:
            if num_blocks is None:
                free, _ = torch.cuda.mem_get_info(self.device)
                num_blocks = int(free * kv_fraction) // kv_bytes_per_page(cfg, self.model.nkv)
            self.cache = torch.zeros(cfg.layers, num_blocks, 2, self.model.nkv, PAGE, cfg.head_dim,
                                     dtype=torch.bfloat16, device=self.device)
        self.alloc = BlockAllocator(num_blocks)
        settings = getattr(self.model, "settings", None)
        self.guard = ServeGuard(self.model, z_alarm=settings.z_alarm if settings is not None else 6.0)
        # every activation buffer and the GEMM workspace are sized once, before any CUDA graph is captured
        self.model.buffers(max(max_prefill_tokens, max_num_seqs))
        self.max_model_len = -(-max_model_len // 256) * 256
        self.model.decode_scratch(max_num_seqs, self.max_model_len)
        self._graphs: dict = {}
        self._graph_kernels: dict = {}     # graph key -> this library's kernels captured in it
        self._graph_replayed = 0           # kernels of this library executed by graph replays
        self.step_counter = 0
        self.stats = {"prefill_tokens": 0, "decode_tokens": 0, "steps": 0}
        self.hooks = None                  # serve.plugin.PluginHooks (register() sets it)
        self.phase_timing = False          # record device time of the prefill and decode phases of generate()
        self.last_phase_ms: dict = {}
        self.tap: Optional[TokenTap] = None   # set during a generate() call that streams its tokens

    def describe(self) -> dict:
        """The engine's configuration as the offline deployment contracts read it (`evidence/config.py`)."""
        from .. import __version__
        return {"engine": "sdcguard_b200", "version": __version__, "model": self.cfg.name,
                "kv_pages": int(self.alloc.num_blocks), "page_tokens": PAGE, "max_num_seqs": self.max_num_seqs,
                "max_model_len": self.max_model_len, "checked": bool(self.checked), "sample_every": self.sample_every,
                "kv_page_bytes": kv_bytes_per_page(self.cfg, self.model.nkv)}

    def startup_line(self) -> str:
        """One line for the startup log: `sdcguard_b200 engine: key=value ...` (parsed by `evidence.config`)."""
        return "sdcguard_b200 engine: " + " ".join(f"{k}={v}" for k, v in self.describe().items())

    # ---------------------------------------------------------------- prefill
    def _prefill_batch(self, reqs: list[int], prompts_dev: torch.Tensor, plens: list[int], bt_dev: torch.Tensor,
                       bt_host: list[list[int]], out_tokens: torch.Tensor) -> None:
        dev = self.device
        toks, pos, slots, starts, lens, last = [], [], [], [], [], []
        t0 = 0
        for r in reqs:
            n = plens[r]
            starts.append(t0)
            lens.append(n)
            pos.extend(range(n))
            pages = bt_host[r]
            slots.extend(pages[p // PAGE] * PAGE + p % PAGE for p in range(n))
            t0 += n
            last.append(t0 - 1)
        T = t0
        rows_req = torch.tensor(reqs, dtype=torch.long)
        tok_dev = torch.cat([prompts_dev[r, :plens[r]] for r in reqs])
        group = self.model.nq // self.model.nkv
        tiles = attention.prefill_tiles(starts, lens, group)
        # the tiles index block-table rows of this batch: gather those rows
        bt_b = bt_dev.index_select(0, rows_req.to(dev))
        meta = StepMeta(
            mode="prefill", tokens=tok_dev,
            pos=torch.tensor(pos, dtype=torch.int32).to(dev, non_blocking=True),
            slots=torch.tensor(slots, dtype=torch.int64).to(dev, non_blocking=True),
            block_table=bt_b, logits_rows=torch.tensor(last, dtype=torch.int64).to(dev, non_blocking=True),
            tiles=tiles.to(dev, non_blocking=True))
        if self.checked:
            # replay sample: per request a run of ceil(n / sample_every) consecutive tokens at an offset that
            # rotates with the step, so successive prefills of a prompt length cover all of it. One run per
            # request makes one replay tile, which attends only to the keys up to the run's end (rows spread over
            # the whole prompt would make the replay read the request's full context).
            samp, per_req = [], []
            for i in range(len(reqs)):
                n = lens[i]
                k = -(-n // self.sample_every)
                o = min(((self.step_counter + i) % self.sample_every) * k, n - k)
                run = list(range(starts[i] + o, starts[i] + o + k))
                samp.extend(run)
                per_req.append(run)
            rt, ridx = attention.replay_tiles(per_req, group)
            meta.sample_rows = torch.tensor(samp, dtype=torch.int32).to(dev, non_blocking=True)
            meta.sample_tiles = rt.to(dev, non_blocking=True)
            meta.sample_idx = ridx.to(dev, non_blocking=True)
        logits = self.model.forward(meta, self.cache)
        nxt = self.model.sample(logits)
        out_tokens.index_put_((rows_req.to(dev), torch.zeros(len(reqs), dtype=torch.long, device=dev)), nxt)
        self.step_counter += 1
        self.stats["prefill_tokens"] += T
        self.stats["steps"] += 1
        if self.hooks is not None:
            self.hooks.after_step("prefill", [reqs[i] for i, n in enumerate(lens) for _ in range(n)])

    # ---------------------------------------------------------------- decode
    def _decode_graph(self, B: int, max_pages: int, max_ctx: int, S: int):
        key = (B, max_pages, max_ctx, S)
        g = self._graphs.get(key)
        if g is not None:
            return g
        dev = self.device
        st = dict(
            tokens=torch.zeros(B, dtype=torch.long, device=dev),
            pos=torch.zeros(B, dtype=torch.int32, device=dev),
            slots=torch.zeros(B, dtype=torch.int64, device=dev),
            ctx=torch.ones(B, dtype=torch.int32, device=dev),
            seq_req=torch.arange(B, dtype=torch.int32, device=dev),
            bt=torch.zeros(B, max_pages, dtype=torch.int32, device=dev),
            rows=torch.arange(B, dtype=torch.long, device=dev),
            sample=torch.zeros(max(S, 1), dtype=torch.int32, device=dev),
        )
        meta = StepMeta(mode="decode", tokens=st["tokens"], pos=st["pos"], slots=st["slots"], block_table=st["bt"],
                        logits_rows=st["rows"], seq_req=st["seq_req"], ctx=st["ctx"], max_ctx=max_ctx,
                        sample_rows=st["sample"] if (self.checked and S > 0) else None)
        self.model.buffers(B)

        def run():
            logits = self.model.forward(meta, self.cache)
            return self.model.sample(logits)

        if not self.cuda_graph:
            g = (None, st, run)
            self._graphs[key] = g
            return g
        # warm up outside the graph (lazy module loading, workspace sizing), on a side stream as capture requires
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            run()
        torch.cuda.current_stream(dev).wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        from .. import _native
        n0 = _native.launch_count()
        with torch.cuda.graph(graph):
            out = run()
        # captured calls are not launches; they run at every replay
        self._graph_kernels[key] = _native.launch_count() - n0
        _native._launches[0] = n0
        g = (graph, st, out)
        self._graphs[key] = g
        return g

    def _decode(self, plens: list[int], bt_dev: torch.Tensor, out_tokens: torch.Tensor, max_new: int) -> None:
        dev = self.device
        N = len(plens)
        for b0 in range(0, N, self.max_num_seqs):
            idx = list(range(b0, min(N, b0 + self.max_num_seqs)))
            B = len(idx)
            max_pages = bt_dev.shape[1]
            max_ctx = max(plens[r] for r in idx) + max_new
            if max_ctx > self.max_model_len:
                raise ValueError(f"sequence of {max_ctx} tokens exceeds max_model_len={self.max_model_len}")
            max_ctx = self.max_model_len
            S = -(-B // self.sample_every) if self.checked else 0
            graph, st, out = self._decode_graph(B, max_pages, max_ctx, S)
            rows = torch.tensor(idx, dtype=torch.long, device=dev)
            st["bt"].copy_(bt_dev.index_select(0, rows))
            pl = torch.tensor([plens[r] for r in idx], dtype=torch.int64, device=dev)
            steps = torch.arange(max_new - 1, dtype=torch.int64, device=dev)
            pos_all = pl[None, :] + steps[:, None]                       # (steps, B)
            pages = st["bt"].long().gather(1, (pos_all // PAGE).t()).t()  # (steps, B)
            slots_all = pages * PAGE + pos_all % PAGE
            samples = []
            for s in range(max_new - 1):
                salt = (self.step_counter + s) % self.sample_every
                sm = [b for b in range(B) if (b + salt) % self.sample_every == 0]
                sm = (sm + sm[:1] * S)[:S] if sm else [0] * S
                samples.append(sm)
            samp_all = torch.tensor(samples, dtype=torch.int32).to(dev) if S else None
            for s in range(max_new - 1):
                st["tokens"].copy_(out_tokens.index_select(0, rows)[:, s])
                st["pos"].copy_(pos_all[s])
                st["slots"].copy_(slots_all[s])
                st["ctx"].copy_(pos_all[s] + 1)
                if S:
                    st["sample"].copy_(samp_all[s])
                if graph is not None:
                    graph.replay()
                    self._graph_replayed += self._graph_kernels[(B, max_pages, max_ctx, S)]
                    nxt = out
                else:
                    nxt = out()
                out_tokens[rows, s + 1] = nxt
                if self.tap is not None:
                    self.tap.push(idx, s + 1, nxt)
                if self.hooks is not None:
                    self.hooks.after_step("decode", idx)
            self.step_counter += max_new - 1
            self.stats["decode_tokens"] += B * (max_new - 1)
            self.stats["steps"] += max_new - 1

    def graph_launches(self) -> int:
        """This library's kernels executed by CUDA-graph replays so far (eager launches are counted by
        sdcguard_b200._native.launch_count)."""
        return self._graph_replayed

    # ---------------------------------------------------------------- public API
    def check_tokens(self, prompts: torch.Tensor, plens: Sequence[int]) -> None:
        """Host-side range check of prompt token ids (an out-of-range id must be an error here, not a device
        assert in the embedding gather)."""
        if prompts.device.type != "cpu":
            return
        for r, n in enumerate(plens):
            row = prompts[r, :n]
            if n and (int(row.min()) < 0 or int(row.max()) >= self.cfg.vocab):
                raise ValueError(f"request {r}: token ids must lie in [0, {self.cfg.vocab})")

    def block_tables(self, pages: Sequence[Sequence[int]]) -> torch.Tensor:
        """(N, max_pages) int32 device block table from per-request page lists."""
        max_pages = max(len(p) for p in pages)
        bt = torch.zeros(len(pages), max_pages, dtype=torch.int32)
        for r, pg in enumerate(pages):
            bt[r, :len(pg)] = torch.tensor(list(pg), dtype=torch.int32)
        return bt.to(self.device, non_blocking=True)

    def prefill(self, prompts_dev: torch.Tensor, plens: Sequence[int], pages: Sequence[Sequence[int]],
                out_tokens: torch.Tensor) -> None:
        """Prefill every request into its pages (token budget per batch) and write each request's first generated
        token to out_tokens[:, 0]. The pages stay allocated (the caller owns them)."""
        plens = [int(x) for x in plens]
        bt_dev = self.block_tables(pages)
        batch, ntok = [], 0
        for r in range(len(plens)):
            if batch and ntok + plens[r] > self.max_prefill_tokens:
                self._prefill_batch(batch, prompts_dev, plens, bt_dev, pages, out_tokens)
                batch, ntok = [], 0
            batch.append(r)
            ntok += plens[r]
        if batch:
            self._prefill_batch(batch, prompts_dev, plens, bt_dev, pages, out_tokens)

    def decode_from(self, plens: Sequence[int], pages: Sequence[Sequence[int]], out_tokens: torch.Tensor,
                    max_new_tokens: int) -> None:
        """Decode max_new_tokens - 1 further tokens for requests whose prompts are already in `pages` and whose
        first token is out_tokens[:, 0] (e.g. KV pages received from a prefill engine)."""
        if max_new_tokens > 1:
            self._decode([int(x) for x in plens], self.block_tables(pages), out_tokens, max_new_tokens)

    def score(self, seqs: Sequence[Sequence[int]], topk: int = 20) -> list[tuple[torch.Tensor, torch.Tensor]]:
        """Teacher-forced log-probabilities: for every sequence, one prefill over all its tokens with logits at every
        position; returns per sequence (values, ids) of the top-k log-softmax entries, (len, topk) on the host.
        Position p's distribution is the prediction of token p + 1. Checks run as in any prefill."""
        dev = self.device
        group = self.model.nq // self.model.nkv
        out = []
        for ids in seqs:
            n = len(ids)
            if n > self.max_prefill_tokens:
                raise ValueError(f"sequence of {n} tokens exceeds max_prefill_tokens {self.max_prefill_tokens}")
            pages = self.alloc.alloc(-(-n // PAGE))
            try:
                meta = StepMeta(
                    mode="prefill", tokens=torch.tensor(list(ids), dtype=torch.long).to(dev),
                    pos=torch.arange(n, dtype=torch.int32).to(dev),
                    slots=torch.tensor([pages[p // PAGE] * PAGE + p % PAGE for p in range(n)], dtype=torch.int64).to(dev),
                    block_table=self.block_tables([pages]), logits_rows=torch.arange(n, dtype=torch.int64).to(dev),
                    tiles=attention.prefill_tiles([0], [n], group).to(dev))
                logits = self.model.forward(meta, self.cache)
                v, i = torch.log_softmax(logits.float(), -1).topk(topk, -1)
                out.append((v.cpu(), i.cpu()))
            finally:
                self.alloc.release(pages)
        return out

    def generate(self, prompts: torch.Tensor, prompt_lens: Sequence[int], max_new_tokens: int,
                 on_tokens: Optional[Callable] = None) -> torch.Tensor:
        """prompts: (N, max_len) int64 token ids (ideally pinned host memory); returns (N, max_new_tokens) int64
        generated ids on the host. Greedy decoding, no early stop (synthetic workloads).

        on_tokens(rows, column, ids): called from a tap thread with each generated column once the GPU has written
        it (column 0 after the prefill, then one per decode step), for streaming responses (TokenTap)."""
        dev = self.device
        N = prompts.shape[0]
        plens = [int(x) for x in prompt_lens]
        self.check_tokens(prompts, plens)
        prompts_dev = prompts.to(dev, non_blocking=True)
        need = [-(-(n + max_new_tokens) // PAGE) for n in plens]
        pages = [self.alloc.alloc(k) for k in need]
        out_tokens = torch.zeros(N, max_new_tokens, dtype=torch.long, device=dev)
        try:
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)] if self.phase_timing else None
            if ev:
                ev[0].record()
            if on_tokens is not None and dev.type == "cuda":
                self.tap = TokenTap(dev, N, max_new_tokens, on_tokens)
            with nvtx_range("sdcguard.prefill"):
                self.prefill(prompts_dev, plens, pages, out_tokens)
            if self.tap is not None:
                self.tap.push(list(range(N)), 0, out_tokens[:, 0])
            if ev:
                ev[1].record()
            with nvtx_range("sdcguard.decode"):
                self.decode_from(plens, pages, out_tokens, max_new_tokens)
            if ev:
                ev[2].record()
            host = torch.empty(N, max_new_tokens, dtype=torch.long, pin_memory=True)
            host.copy_(out_tokens, non_blocking=True)
            torch.cuda.current_stream(dev).synchronize()
            if ev:
                self.last_phase_ms = {"prefill": ev[0].elapsed_time(ev[1]), "decode": ev[1].elapsed_time(ev[2])}
            if self.tap is not None:
                tap, self.tap = self.tap, None
                tap.close()
            return host
        finally:
            if self.tap is not None:
                tap, self.tap = self.tap, None
                tap.q.put(None)
            for pg in pages:
                self.alloc.release(pg)
