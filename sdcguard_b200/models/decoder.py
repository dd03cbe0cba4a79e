"""Decoder-only transformer (Llama / Qwen3 family) running on this library's sm_100a kernels, with every
GEMM checked by the fused ABFT epilogue and the other ops checked by exact replay of a rotating sample of rows.

Per layer (rows = tokens of the batch):
    h, y  = add_rmsnorm(prev, h)                    replay-checked on sampled rows
    qkv   = checked GEMM  y @ Wqkv^T                ABFT, every row
    q,k,v = qk_norm + RoPE, k/v -> paged cache      replay in compare mode (q bits, cache bits, slot mapping)
    o     = paged attention (prefill or decode)      replay-checked on sampled rows
    a     = checked GEMM  o @ Wo^T                  ABFT
    h, y2 = add_rmsnorm(a, h)                       replay-checked
    gu    = checked GEMM  y2 @ Wgu^T                ABFT
    act   = silu(g) * u                             replay-checked
    out   = checked GEMM  act @ Wdown^T             ABFT
then the final norm and the checked LM-head GEMM on the rows whose next token is needed.

`checked=False` runs the same model with cuBLAS GEMMs (torch.matmul) and no checks: the unchecked baseline.

Weights are random (N(0, 0.02) for matrices, ones for norms): the benchmarks use synthetic data of the named
shapes. Reference: the guarded serving path of src/sdcguard/serve.py (ServeGuard.attach / check_static) and the
vLLM integration points of src/sdcguard/vllm_plugin.py:2315-2501; here the model itself is the engine.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import torch

from ..ops import attention, spot, gemm, layers


@dataclass(frozen=True)
class DecoderConfig:
    name: str
    layers: int
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    rope_theta: float
    rms_eps: float
    qk_norm: bool
    tie_embeddings: bool = False
    rope_scaling: Optional[dict] = None
    max_position: int = 8192


QWEN3_0_6B = DecoderConfig("Qwen3-0.6B", 28, 1024, 16, 8, 128, 3072, 151936, 1_000_000.0, 1e-6, True,
                           tie_embeddings=True, max_position=40960)
LLAMA3_8B = DecoderConfig("Llama-3-8B", 32, 4096, 32, 8, 128, 14336, 128256, 500_000.0, 1e-5, False,
                          rope_scaling=None, max_position=8192)
TINY = DecoderConfig("tiny", 2, 256, 4, 2, 128, 512, 1024, 10_000.0, 1e-6, True, max_position=4096)

CONFIGS = {c.name: c for c in (QWEN3_0_6B, LLAMA3_8B, TINY)}


@dataclass
class StepMeta:
    """Device-side description of one forward step (prefill batch or decode step)."""
    mode: str                         # "prefill" or "decode"
    tokens: torch.Tensor              # (T,) int64 input ids
    pos: torch.Tensor                 # (T,) int32 positions
    slots: torch.Tensor               # (T,) int64 KV slots (block * 16 + offset)
    block_table: torch.Tensor         # (R, max_pages) int32
    logits_rows: torch.Tensor         # (L,) int64 rows whose next token is computed
    tiles: Optional[torch.Tensor] = None        # prefill tiles (n, 4) int32
    seq_req: Optional[torch.Tensor] = None      # decode: (B,) int32 block-table row
    ctx: Optional[torch.Tensor] = None          # decode: (B,) int32 keys per sequence
    max_ctx: int = 0
    # replay sample (checked mode): rows and their attention replay description
    sample_rows: Optional[torch.Tensor] = None  # (S,) int32
    sample_tiles: Optional[torch.Tensor] = None  # prefill replay tiles
    sample_idx: Optional[torch.Tensor] = None   # prefill replay token list (same rows, tile order)


def _init_linear(n: int, k: int, gen: torch.Generator, device) -> torch.Tensor:
    w = torch.empty(n, k, dtype=torch.float32, device="cpu").normal_(0.0, 0.02, generator=gen)
    return w.to(device=device, dtype=torch.bfloat16)


@dataclass
class LayerWeights:
    ln1: torch.Tensor
    ln2: torch.Tensor
    qkv: torch.Tensor
    o: torch.Tensor
    gate_up: torch.Tensor
    down: torch.Tensor
    q_norm: Optional[torch.Tensor] = None
    k_norm: Optional[torch.Tensor] = None
    cw: dict = field(default_factory=dict)   # name -> gemm.CheckedWeight


class CheckedDecoder:
    """The model plus its check state. Slots of the state table name each checked op (`state.names`)."""

    def __init__(self, cfg: DecoderConfig, device="cuda", checked: bool = True, seed: int = 0,
                 weights: Optional[dict] = None, tp_rank: int = 0, tp_size: int = 1, moe_layers: Optional[list] = None,
                 precision: str = "bf16", settings=None):
        """moe_layers: one `models.moe.MoELayer` per layer in place of the dense MLP (expert-parallel models).
        precision "fp8": the four projections of every layer run on the block-scaled fp8 checked GEMM (activations
        quantized per call with 1 x 128 scales, replay-checked on the sampled rows); the LM head stays bf16."""
        if precision not in ("bf16", "fp8"):
            raise ValueError("precision must be bf16 or fp8")
        if precision == "fp8" and not checked:
            raise ValueError("the fp8 path is the checked fp8 GEMM")
        self.precision = precision
        from ..serve.settings import CheckSettings
        self.settings = settings if settings is not None else CheckSettings.from_env()
        self._side = torch.cuda.Stream(torch.device(device)) if checked and torch.cuda.is_available() else None
        self.cfg = cfg
        self.moe = moe_layers
        self.device = torch.device(device)
        self.checked = checked
        self.nq = cfg.heads // tp_size
        self.nkv = max(1, cfg.kv_heads // tp_size)
        self.inter = cfg.intermediate // tp_size
        d = cfg.head_dim
        gen = torch.Generator().manual_seed(seed)
        dev = self.device
        self.embed = _init_linear(cfg.vocab, cfg.hidden, gen, dev)
        self.final_ln = torch.ones(cfg.hidden, dtype=torch.bfloat16, device=dev)
        self.lm_head = self.embed if cfg.tie_embeddings else _init_linear(cfg.vocab, cfg.hidden, gen, dev)
        self.layers: list[LayerWeights] = []
        for _ in range(cfg.layers):
            lw = LayerWeights(
                ln1=torch.ones(cfg.hidden, dtype=torch.bfloat16, device=dev),
                ln2=torch.ones(cfg.hidden, dtype=torch.bfloat16, device=dev),
                qkv=_init_linear((self.nq + 2 * self.nkv) * d, cfg.hidden, gen, dev),
                o=_init_linear(cfg.hidden, self.nq * d, gen, dev),
                gate_up=None if moe_layers else _init_linear(2 * self.inter, cfg.hidden, gen, dev),
                down=None if moe_layers else _init_linear(cfg.hidden, self.inter, gen, dev),
                q_norm=torch.ones(d, dtype=torch.bfloat16, device=dev) if cfg.qk_norm else None,
                k_norm=torch.ones(d, dtype=torch.bfloat16, device=dev) if cfg.qk_norm else None,
            )
            self.layers.append(lw)
        self.rope = layers.rope_table(min(cfg.max_position, 16384), d, cfg.rope_theta, cfg.rope_scaling, device=dev)
        self.state = gemm.StateTable(dev, 16 * cfg.layers + 8)
        self.slot: dict[str, int] = {}
        if precision == "fp8":
            from ..ops.fp8 import Fp8Linears
            self.fp8 = Fp8Linears(dev)
        self.spot_schedules: dict = {}
        self._spot_turn = 0
        self.slot_weights: dict = {}       # state slot -> CheckedWeight (the float64 recheck of a captured alarm)
        if checked:
            for i, lw in enumerate(self.layers):
                for p_i, name in enumerate(("qkv", "o", "gate_up", "down")):
                    if getattr(lw, name) is None:
                        continue
                    if precision == "bf16" and not self.settings.gemm_checked(i, p_i):
                        continue       # outside this replica's share: runs unchecked on the library GEMM
                    if precision == "fp8":
                        fw = self.fp8.add(f"L{i}.{name}", getattr(lw, name))
                        self.slot[f"L{i}.{name}"] = self.state.add(f"layers.{i}.{name} (ABFT fp8 GEMM)", fw.nb)
                        self.slot[f"L{i}.{name}.q"] = self.state.add(f"layers.{i}.{name}.quant (replay)", 1)
                        continue
                    cw = gemm.CheckedWeight(getattr(lw, name))
                    lw.cw[name] = cw
                    self.slot[f"L{i}.{name}"] = self.state.add(f"layers.{i}.{name} (ABFT GEMM)", cw.nb)
                    self.slot_weights[self.slot[f"L{i}.{name}"]] = cw
                    if self.settings.spot:
                        self.slot[f"L{i}.{name}.spot"] = self.state.add(f"layers.{i}.{name} (spot check)",
                                                                         getattr(lw, name).shape[0], "rowblock")
                        self.spot_schedules[f"L{i}.{name}"] = spot.SpotSchedule(getattr(lw, name).shape[0])
                for name in ("norm1", "rope_kv", "attn", "norm2", "act"):
                    self.slot[f"L{i}.{name}"] = self.state.add(f"layers.{i}.{name} (replay)", 1)
            self.lm_cw = gemm.CheckedWeight(self.lm_head)
            self.slot["lm_head"] = self.state.add("lm_head (ABFT GEMM)", self.lm_cw.nb)
            self.slot_weights[self.slot["lm_head"]] = self.lm_cw
            self.slot["final_norm"] = self.state.add("final_norm (replay)", 1)
        if moe_layers:
            for i, m in enumerate(moe_layers):
                m.attach(self.state, f"layers.{i}.moe")
            comm = moe_layers[0].comm
            if checked:
                d = self.state.add("ep dispatch (transfer seals)", comm.nb, "rowblock")
                c = self.state.add("ep combine (transfer seals)", comm.nb, "rowblock")
                assert c == d + 1
                comm.state = self.state.state[d:d + 2]
        self._bufs: dict = {}

    # ---------------------------------------------------------------- buffers
    def buffers(self, T: int) -> dict:
        """Scratch activations for up to T rows, reused across steps (views keep their data pointers)."""
        b = self._bufs.get("cap", 0)
        if T <= b:
            return self._bufs
        cfg, dev, bf = self.cfg, self.device, torch.bfloat16
        H, D = cfg.hidden, cfg.head_dim
        nq, nkv = self.nq, self.nkv
        self._bufs = dict(
            cap=T,
            x=torch.empty(T, H, dtype=bf, device=dev),
            resid=torch.empty(T, H, dtype=bf, device=dev),
            y=torch.empty(T, H, dtype=bf, device=dev),
            rs=torch.empty(T, dtype=torch.float32, device=dev),
            qkv=torch.empty(T, (nq + 2 * nkv) * D, dtype=bf, device=dev),
            q=torch.empty(T, nq, D, dtype=bf, device=dev),
            attn=torch.empty(T, nq, D, dtype=bf, device=dev),
            ors=torch.empty(T, dtype=torch.float32, device=dev),
            a=torch.empty(T, H, dtype=bf, device=dev),
            gu=torch.empty(T if not self.moe else 1, 2 * self.inter, dtype=bf, device=dev),
            act=torch.empty(T if not self.moe else 1, self.inter, dtype=bf, device=dev),
        )
        if self.precision == "fp8":
            self.fp8.reserve(T, max(H, nq * D, self.inter))
        if self.checked:
            gemm.reserve_workspace(dev, T, max(2 * self.inter if not self.moe else 0, (nq + 2 * nkv) * D, H))
            gemm.reserve_workspace(dev, min(T, 1024), cfg.vocab)
        return self._bufs

    def _side_stream(self) -> torch.cuda.Stream:
        """The stream replay checks run on (created once, before any graph capture needs it)."""
        if getattr(self, "_side", None) is None:
            self._side = torch.cuda.Stream(self.device)
        return self._side

    def decode_scratch(self, nseq: int, max_ctx: int) -> torch.Tensor:
        """Split-KV partials for decode; sized once for the largest batch and context seen (graph-safe: a decode
        graph is captured after the engine reserved it)."""
        key = (nseq, max_ctx)
        cur = self._bufs.get("dscratch")
        need = attention.decode_scratch(nseq, self.nq, self.nkv, max_ctx, "meta").numel()
        if cur is None or cur.numel() < need:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("decode scratch too small inside graph capture")
            self._bufs["dscratch"] = torch.empty(need, dtype=torch.float32, device=self.device)
        return self._bufs["dscratch"]

    # ---------------------------------------------------------------- ops
    def inject_next(self, name: str, row: int, col: int, xor_bits: int) -> None:
        """Fault injection: the next eager (not graph-captured) bf16 GEMM of layer `name` (e.g. "L0.down") flips
        `xor_bits` of its fp32 accumulator (row, col) before the check and the rounding."""
        self._inject = (name, (row, col, xor_bits))

    def _linear(self, x, w, cw, name, out, row_sq, sample=None):
        if self.precision == "fp8":
            return self.fp8.linear(name, x, self.state.state, self.slot[name], out,
                                   qcheck=self.state.state[self.slot[name + ".q"]], sample=sample)
        if not self.checked or (self.precision == "bf16" and name not in self.slot):
            return torch.matmul(x, w.t(), out=out)
        inj = None
        if getattr(self, "_inject", None) and self._inject[0] == name and \
                not torch.cuda.is_current_stream_capturing():
            inj, self._inject = self._inject[1], None
        return gemm.checked_linear(x, cw, self.state.state, self.slot[name], row_sq=row_sq, out=out, inject=inj)

    def _st(self, name) -> torch.Tensor:
        return self.state.state[self.slot[name]]

    def _next_spot_target(self, lo: int, hi: int):
        """The projection the spot check recomputes in this step: the registered ones take turns."""
        names = [n for n in self.spot_schedules if lo <= int(n[1:].split(".")[0]) < hi]
        if not names:
            return None
        self._spot_turn += 1
        return names[self._spot_turn % len(names)]

    def _spot(self, name: str, x: torch.Tensor, w: torch.Tensor, y: torch.Tensor, T: int) -> None:
        sched = self.spot_schedules[name]
        rows, cols = sched.sample(T, self._spot_turn // max(1, len(self.spot_schedules)), self.device)
        spot.spot_check(x, w, y, rows, cols, self._st(name + ".spot"))

    def forward(self, meta: StepMeta, cache: torch.Tensor, layer_range: Optional[tuple] = None,
                hidden: Optional[tuple] = None, last: bool = True):
        """Runs one step; returns logits (L, vocab) bf16 for meta.logits_rows. cache: (layers, blocks, 2, nkv,
        16, 128) bf16. Pipeline stages: layer_range=(lo, hi) runs only those layers (cache then holds hi - lo layers),
        hidden=(x, resid) enters after layer lo - 1 instead of the embedding, and last=False returns the (x, resid)
        pair after layer hi - 1 (x: the last sublayer's output, not yet added to the residual resid)."""
        cfg = self.cfg
        T = meta.tokens.shape[0]
        B = self.buffers(T)
        x, resid, y, rs = B["x"][:T], B["resid"][:T], B["y"][:T], B["rs"][:T]
        qkv, q, att, ors = B["qkv"][:T], B["q"][:T], B["attn"][:T], B["ors"][:T]
        a, gu, act = B["a"][:T], B["gu"][:T], B["act"][:T]
        lo, hi = layer_range or (0, len(self.layers))
        if hidden is None:
            torch.index_select(self.embed, 0, meta.tokens, out=x)
        else:
            x.copy_(hidden[0])
            resid.copy_(hidden[1])
        S = meta.sample_rows
        chk = self.checked and S is not None and S.numel() > 0
        st = self.settings
        spot_on = self.checked and st.spot and meta.mode == "prefill" and self.precision == "bf16" and T > 0
        spot_target = self._next_spot_target(lo, hi) if spot_on else None
        nq, nkv, D = self.nq, self.nkv, cfg.head_dim
        # Replay checks write nothing the forward reads, so they run on a side stream next to the main chain (filling
        # SMs the small decode kernels leave idle) and rejoin before the buffers they compare are overwritten: the
        # norm-1 / rope / attention replays before norm 2 of the same layer, the norm-2 / SwiGLU replays before the
        # next layer's norm 1.
        main = torch.cuda.current_stream(self.device)
        side = self._side_stream() if (chk or spot_target is not None) else None
        forked = [False]      # joined only after a fork: under graph capture the side stream must be in the capture

        def replay(fn):
            if side is None:
                fn()
                return
            side.wait_stream(main)
            forked[0] = True
            with torch.cuda.stream(side):
                fn()

        def join():
            if side is not None and forked[0]:
                main.wait_stream(side)
                forked[0] = False

        for i in range(lo, hi):
            join()
            lw = self.layers[i]
            lc = cache[i - lo]
            if i == 0:
                layers.add_rmsnorm(x, lw.ln1, cfg.rms_eps, residual=None, resid_out=resid, out=y, row_sq=rs)
            else:
                layers.add_rmsnorm(x, lw.ln1, cfg.rms_eps, residual=resid, resid_out=resid, out=y, row_sq=rs)
            if chk and st.norms:
                replay(lambda: layers.add_rmsnorm(resid, lw.ln1, cfg.rms_eps, out=y, rows=S,
                                                  check=self._st(f"L{i}.norm1")))
            self._linear(y, lw.qkv, lw.cw.get("qkv"), f"L{i}.qkv", qkv, rs, S)
            if spot_target == f"L{i}.qkv":
                replay(lambda: self._spot(f"L{i}.qkv", y, lw.qkv, qkv, T))
            layers.qk_norm_rope_kv(qkv, nq, nkv, meta.pos, meta.slots, lw.q_norm, lw.k_norm, cfg.rms_eps, self.rope,
                                   q, lc)
            if chk and st.rope:
                replay(lambda: layers.qk_norm_rope_kv(qkv, nq, nkv, meta.pos, meta.slots, lw.q_norm, lw.k_norm,
                                                      cfg.rms_eps, self.rope, q, lc, rows=S,
                                                      check=self._st(f"L{i}.rope_kv")))
            ors.zero_()
            if meta.mode == "prefill":
                attention.prefill(q, lc, meta.block_table, meta.pos, meta.tiles, nq, nkv, out=att, row_sq=ors)
                if chk and st.attn:
                    replay(lambda: attention.prefill(q, lc, meta.block_table, meta.pos, meta.sample_tiles, nq, nkv,
                                                     out=att, row_idx=meta.sample_idx, check=self._st(f"L{i}.attn")))
            else:
                scratch = self.decode_scratch(T, meta.max_ctx)
                attention.decode(q, lc, meta.block_table, meta.seq_req, meta.ctx, nq, nkv, meta.max_ctx, out=att,
                                 row_sq=ors, scratch=scratch)
                if chk and st.attn:
                    replay(lambda: attention.decode(q, lc, meta.block_table, meta.seq_req, meta.ctx, nq, nkv,
                                                    meta.max_ctx, out=att, seq_idx=S, scratch=scratch,
                                                    check=self._st(f"L{i}.attn")))
            self._linear(att.view(T, nq * D), lw.o, lw.cw.get("o"), f"L{i}.o", a, ors, S)
            if spot_target == f"L{i}.o":
                replay(lambda: self._spot(f"L{i}.o", att.view(T, nq * D), lw.o, a, T))
            join()
            layers.add_rmsnorm(a, lw.ln2, cfg.rms_eps, residual=resid, resid_out=resid, out=y, row_sq=rs)
            if chk and st.norms:
                replay(lambda: layers.add_rmsnorm(resid, lw.ln2, cfg.rms_eps, out=y, rows=S,
                                                  check=self._st(f"L{i}.norm2")))
            if self.moe:
                x = self.moe[i].forward(y, S if chk else None)
                continue
            self._linear(y, lw.gate_up, lw.cw.get("gate_up"), f"L{i}.gate_up", gu, rs, S)
            if spot_target == f"L{i}.gate_up":
                replay(lambda: self._spot(f"L{i}.gate_up", y, lw.gate_up, gu, T))
            layers.silu_mul(gu, out=act, row_sq=rs)
            if chk and st.act:
                replay(lambda: layers.silu_mul(gu, out=act, rows=S, check=self._st(f"L{i}.act")))
            self._linear(act, lw.down, lw.cw.get("down"), f"L{i}.down", x, rs, S)
            if spot_target == f"L{i}.down":
                replay(lambda: self._spot(f"L{i}.down", act, lw.down, x, T))
        join()
        if not last:
            return x, resid
        # final norm on the rows that produce tokens, then the LM head
        L = meta.logits_rows.shape[0]
        xs = x.index_select(0, meta.logits_rows)
        rsd = resid.index_select(0, meta.logits_rows)
        yl, rsl = layers.add_rmsnorm(xs, self.final_ln, cfg.rms_eps, residual=rsd, resid_out=rsd)
        if self.checked:
            one = torch.zeros(1, dtype=torch.int32, device=self.device)
            layers.add_rmsnorm(rsd, self.final_ln, cfg.rms_eps, out=yl, rows=one, check=self._st("final_norm"))
        logits = torch.empty(L, cfg.vocab, dtype=torch.bfloat16, device=self.device)
        if self.checked:
            gemm.checked_linear(yl, self.lm_cw, self.state.state, self.slot["lm_head"], row_sq=rsl, out=logits)
        else:
            torch.matmul(yl, self.lm_head.t(), out=logits)
        return logits

    def read_checks(self, reset: bool = False) -> list[dict]:
        return self.state.read(reset=reset)

    def check_coverage(self) -> dict:
        """Which linear layers carry the ABFT check: counts of checked and unchecked projections (the LM head
        included), the share of linear-layer weight elements that are checked, and how many of the checked ones are
        fp8 layers (each with its quantization replay)."""
        checked = unchecked = fp8 = 0
        w_checked = w_total = 0
        for i, lw in enumerate(self.layers):
            for name in ("qkv", "o", "gate_up", "down"):
                w = getattr(lw, name)
                if w is None:
                    continue
                w_total += w.numel()
                if f"L{i}.{name}" in self.slot:
                    checked += 1
                    w_checked += w.numel()
                    fp8 += f"L{i}.{name}.q" in self.slot
                else:
                    unchecked += 1
        w_total += self.lm_head.numel()
        if "lm_head" in self.slot:
            checked += 1
            w_checked += self.lm_head.numel()
        else:
            unchecked += 1
        return {"layers_checked": checked, "layers_unchecked": unchecked, "fp8_layers_checked": fp8,
                "weights_checked_ratio": w_checked / w_total if w_total else 0.0}

    def sample(self, logits: torch.Tensor) -> torch.Tensor:
        """Greedy next token (the engine's sampler)."""
        return torch.argmax(logits, dim=-1)
