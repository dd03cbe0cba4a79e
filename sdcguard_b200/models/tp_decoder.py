"""Tensor-parallel decoder (Megatron-style column/row parallel with sequence parallelism) on this library's checked
GEMMs and checksummed NVLink collectives. Drop-in model for `serve.engine.LLMEngine` (same `forward(meta, cache)`
contract); every rank runs the same engine on the same requests and owns 1/world of the heads, of the MLP and of
the vocabulary, and the rows [rank R, (rank+1) R) of the residual stream.

Per layer:
    y_shard   = RMSNorm(x_shard + residual)            -> written straight into the all-gather source buffer
    y         = all_gather(y_shard)                    seal-checked per (row, block)
    qkv       = checked GEMM  y @ Wqkv_local^T         ABFT; local heads only
    attention on the local heads (paged KV cache of the local kv heads)
    partial   = checked GEMM  o @ Wo_local^T           ABFT; output and seals straight into the symmetric buffer
    a_shard   = reduce_scatter(partial)                seal-checked transit + linearity-checked sum
    ... the same for the MLP (gate_up column-parallel, down row-parallel)
LM head: vocabulary-parallel over the gathered final rows; the token is the arg-max over ranks (a tiny NCCL
all-gather of (max, index) pairs).

`collective="nccl"` with `checked=False` is the baseline: cuBLAS GEMMs and NCCL all-gather / reduce-scatter.

Reference: the reference checks each TP rank's local shard and the row-parallel partial before the all-reduce
(src/sdcguard/guard.py:343-419, _compiled.py:111-155) and does not touch the collectives; here the collective
transit and the reduction are checked too.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from ..ops import attention, gemm, layers
from ..parallel.tp import TPComm, all_gather_nccl, reduce_scatter_nccl
from .decoder import DecoderConfig, LayerWeights, StepMeta


class TPDecoder:
    def __init__(self, cfg: DecoderConfig, comm: Optional[TPComm], rank: int, world: int, device, checked: bool = True,
                 collective: str = "own", max_rows: int = 8192, seed: int = 0, precision: str = "bf16"):
        """precision "fp8": the four projections run on the block-scaled fp8 checked GEMM (see models.decoder)."""
        if precision not in ("bf16", "fp8") or (precision == "fp8" and not checked):
            raise ValueError("precision must be bf16, or fp8 with checked=True")
        self.precision = precision
        if cfg.heads % world or cfg.intermediate % world or cfg.vocab % world:
            raise ValueError("heads, intermediate size and vocabulary must divide by the TP size")
        self.cfg, self.rank, self.world = cfg, rank, world
        self.device = torch.device(device)
        self.checked = checked
        self.collective = collective
        self.comm = comm
        self.nq = cfg.heads // world
        self.nkv = max(1, cfg.kv_heads // world)
        self.inter = cfg.intermediate // world
        self.vocab_l = cfg.vocab // world
        self.max_rows = max_rows
        d, H = cfg.head_dim, cfg.hidden
        dev = self.device
        self.seed = seed
        self.chunks = cfg.kv_heads          # weights are generated in kv_heads chunks: any TP size that divides it
        if self.chunks % world:             # builds the same global model
            raise ValueError(f"TP size {world} must divide the number of KV heads ({cfg.kv_heads})")
        mine = range(rank * self.chunks // world, (rank + 1) * self.chunks // world)
        qh, ih, vh = cfg.heads // self.chunks, cfg.intermediate // self.chunks, cfg.vocab // self.chunks
        self.embed = self._gen("embed", 0, (cfg.vocab, H))                        # replicated
        self.final_ln = torch.ones(H, dtype=torch.bfloat16, device=dev)
        self.lm_head = torch.cat([self._gen("lm_head", c, (vh, H)) for c in mine])
        self.layers: list[LayerWeights] = []
        for i in range(cfg.layers):
            qkv = [self._gen(f"L{i}.qkv", c, ((qh + 2) * d, H)) for c in mine]     # per chunk: q heads, k, v
            gu = [self._gen(f"L{i}.gate_up", c, (2 * ih, H)) for c in mine]       # per chunk: gate rows, up rows
            self.layers.append(LayerWeights(
                ln1=torch.ones(H, dtype=torch.bfloat16, device=dev), ln2=torch.ones(H, dtype=torch.bfloat16, device=dev),
                qkv=torch.cat([w[:qh * d] for w in qkv] + [w[qh * d:(qh + 1) * d] for w in qkv]
                              + [w[(qh + 1) * d:] for w in qkv]),
                o=torch.cat([self._gen(f"L{i}.o", c, (H, qh * d)) for c in mine], dim=1),
                gate_up=torch.cat([w[:ih] for w in gu] + [w[ih:] for w in gu]),
                down=torch.cat([self._gen(f"L{i}.down", c, (H, ih)) for c in mine], dim=1),
                q_norm=torch.ones(d, dtype=torch.bfloat16, device=dev) if cfg.qk_norm else None,
                k_norm=torch.ones(d, dtype=torch.bfloat16, device=dev) if cfg.qk_norm else None))
            del qkv, gu
        self.rope = layers.rope_table(min(cfg.max_position, 16384), d, cfg.rope_theta, cfg.rope_scaling, device=dev)
        self.state = gemm.StateTable(dev, 16 * cfg.layers + 16)
        self.slot: dict[str, int] = {}
        if precision == "fp8":
            from ..ops.fp8 import Fp8Linears
            self.fp8 = Fp8Linears(dev)
        if checked:
            for i, lw in enumerate(self.layers):
                for name in ("qkv", "o", "gate_up", "down"):
                    if precision == "fp8":
                        fw = self.fp8.add(f"L{i}.{name}", getattr(lw, name))
                        self.slot[f"L{i}.{name}"] = self.state.add(f"layers.{i}.{name} (ABFT fp8 GEMM, tp{rank})", fw.nb)
                        self.slot[f"L{i}.{name}.q"] = self.state.add(f"layers.{i}.{name}.quant (replay, tp{rank})", 1)
                        continue
                    cw = gemm.CheckedWeight(getattr(lw, name))
                    lw.cw[name] = cw
                    self.slot[f"L{i}.{name}"] = self.state.add(f"layers.{i}.{name} (ABFT GEMM, tp{rank})", cw.nb)
                for name in ("norm1", "rope_kv", "attn", "norm2", "act"):
                    self.slot[f"L{i}.{name}"] = self.state.add(f"layers.{i}.{name} (replay, tp{rank})", 1)
            self.lm_cw = gemm.CheckedWeight(self.lm_head)
            self.slot["lm_head"] = self.state.add(f"lm_head (ABFT GEMM, tp{rank})", self.lm_cw.nb)
            self.slot["final_norm"] = self.state.add(f"final_norm (replay, tp{rank})", 1)
            if comm is not None and collective == "own":
                # the collective kernels fold their seal / linearity results into two rows of this table
                nb = comm.nb
                rs = self.state.add(f"reduce_scatter (collective: seals + linearity, tp{rank})", nb, "collective")
                ag = self.state.add(f"all_gather (collective: seals, tp{rank})", nb, "collective")
                assert ag == rs + 1
                comm.state = self.state.state[rs:rs + 2]
        self._bufs: dict = {}

    def _gen(self, name: str, chunk: int, shape) -> torch.Tensor:
        """N(0, 0.02) bf16 weights of one chunk, from a generator keyed by (seed, name, chunk) on the device: the
        same chunk has the same values whatever the TP size."""
        key = (self.seed * 1_000_003 + sum(ord(ch) * 131 ** j for j, ch in enumerate(name)) * 257 + chunk) % (2 ** 63)
        g = torch.Generator(device=self.device).manual_seed(key)
        w = torch.empty(shape, dtype=torch.float32, device=self.device).normal_(0.0, 0.02, generator=g)
        return w.to(torch.bfloat16)

    # ------------------------------------------------------------------ engine contract
    def buffers(self, T: int) -> dict:
        T = -(-T // self.world) * self.world
        if T <= self._bufs.get("cap", 0):
            return self._bufs
        cfg, dev, bf = self.cfg, self.device, torch.bfloat16
        H, D, R = cfg.hidden, cfg.head_dim, T // self.world
        self._bufs = dict(cap=T, yfull=torch.empty(T, H, dtype=bf, device=dev), rs=torch.empty(T, dtype=torch.float32,
                          device=dev), qkv=torch.empty(T, (self.nq + 2 * self.nkv) * D, dtype=bf, device=dev),
                          q=torch.empty(T, self.nq, D, dtype=bf, device=dev),
                          att=torch.empty(T, self.nq, D, dtype=bf, device=dev),
                          ors=torch.empty(T, dtype=torch.float32, device=dev),
                          gu=torch.empty(T, 2 * self.inter, dtype=bf, device=dev),
                          act=torch.empty(T, self.inter, dtype=bf, device=dev),
                          xs=torch.empty(R, H, dtype=bf, device=dev), resid=torch.empty(R, H, dtype=bf, device=dev),
                          ys=torch.empty(R, H, dtype=bf, device=dev), rss=torch.empty(R, dtype=torch.float32, device=dev),
                          part=torch.empty(T, H, dtype=bf, device=dev))
        if self.precision == "fp8":
            self.fp8.reserve(T, max(H, self.nq * D, self.inter))
        if self.checked:
            gemm.reserve_workspace(dev, T, max(2 * self.inter, H, (self.nq + 2 * self.nkv) * D))
            gemm.reserve_workspace(dev, min(T, 1024), self.vocab_l)
        return self._bufs

    def decode_scratch(self, nseq: int, max_ctx: int) -> torch.Tensor:
        need = attention.decode_scratch(nseq, self.nq, self.nkv, max_ctx, "meta").numel()
        cur = self._bufs.get("dscratch")
        if cur is None or cur.numel() < need:
            self._bufs["dscratch"] = torch.empty(need, dtype=torch.float32, device=self.device)
        return self._bufs["dscratch"]

    def read_checks(self, reset: bool = False) -> list[dict]:
        return self.state.read(reset=reset)

    # ------------------------------------------------------------------ pieces
    def _linear(self, x, w, cw, name, out, row_sq, seal=None, sample=None):
        if self.precision == "fp8":
            y = self.fp8.linear(name, x, self.state.state, self.slot[name], out,
                                qcheck=self.state.state[self.slot[name + ".q"]], sample=sample)
            if seal is not None:
                from ..parallel.tp import seal_rows
                seal_rows(y, seal)
            return y
        if not self.checked:
            return torch.matmul(x, w.t(), out=out)
        return gemm.checked_linear(x, cw, self.state.state, self.slot[name], row_sq=row_sq, out=out, seal=seal)

    def _ag(self, shard_src: torch.Tensor, R: int, out: torch.Tensor,
            rs_out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """All-gather of the shards; with own collectives the shard norm already sealed and signalled them, and
        rs_out (when given) receives the gathered row_sq the next checked GEMM needs."""
        if self.collective == "own":
            return self.comm.all_gather(R, out, rs_out=rs_out, sealed=True)
        return all_gather_nccl(shard_src, out)

    def _norm_into_shard(self, x, w, residual, R):
        """RMSNorm of this rank's rows, written where the all-gather reads them (own collectives: one kernel that
        also seals the shard, writes its row_sq and signals the peers)."""
        B = self._bufs
        if self.collective == "own":
            return self.comm.norm_shard(x, w, self.cfg.rms_eps, residual, B["resid"][:R], R)
        dst = B["ys"][:R]
        layers.add_rmsnorm(x, w, self.cfg.rms_eps, residual=residual, resid_out=B["resid"][:R], out=dst,
                           row_sq=B["rss"][:R])
        return dst

    def _gather_rows(self, ys, R, yfull, rs):
        """All-gather, and the gathered rows' row_sq for the next checked bf16 GEMM (None otherwise)."""
        want = self.checked and self.precision == "bf16"
        if self.collective == "own":
            self._ag(ys, R, yfull, rs_out=rs if want else None)
            return rs if want else None
        self._ag(ys, R, yfull)
        return gemm.row_sqnorm(yfull, out=rs) if want else None

    def _rowpar(self, x, w, cw, name, T, R, row_sq, out_shard, sample=None):
        """Row-parallel GEMM + reduce-scatter into out_shard (R, H)."""
        if (self.collective == "own" and self.checked and self.precision == "bf16" and self.comm.can_push(T)
                and T > 256):
            # one kernel does the GEMM and the transfer (tiles pushed to their owners), then a local reduce
            return self.comm.gemm_reduce_scatter(x, cw, self.state.state, self.slot[name], out_shard, row_sq=row_sq)
        if self.collective == "own":
            self._linear(x, w, cw, name, self.comm.partial(T), row_sq,
                         seal=self.comm.partial_seal(T) if self.checked else None, sample=sample)
            if not self.checked:
                from ..parallel.tp import seal_rows
                seal_rows(self.comm.partial(T), self.comm.partial_seal(T))
            return self.comm.reduce_scatter(T, out_shard)
        part = self._bufs["part"][:T]
        self._linear(x, w, cw, name, part, row_sq)
        return reduce_scatter_nccl(part, out_shard)

    def _st(self, name) -> torch.Tensor:
        return self.state.state[self.slot[name]]

    def _norm_replay(self, ys, w, R, S_loc, name):
        layers.add_rmsnorm(self._bufs["resid"][:R], w, self.cfg.rms_eps, out=ys, rows=S_loc, check=self._st(name))

    def forward(self, meta: StepMeta, cache: torch.Tensor) -> torch.Tensor:
        cfg = self.cfg
        T0 = meta.tokens.shape[0]
        W = self.world
        T = -(-T0 // W) * W
        R = T // W
        B = self.buffers(T)
        dev = self.device
        if T != T0:                      # pad to a multiple of the TP size: pad rows write no KV, attend to nothing
            pad = T - T0
            meta = StepMeta(**{**meta.__dict__,
                               "tokens": torch.cat([meta.tokens, torch.zeros(pad, dtype=torch.long, device=dev)]),
                               "pos": torch.cat([meta.pos, torch.zeros(pad, dtype=torch.int32, device=dev)]),
                               "slots": torch.cat([meta.slots, torch.full((pad,), -1, dtype=torch.long, device=dev)])})
        nq, nkv, D = self.nq, self.nkv, cfg.head_dim
        xs, yfull, rs = B["xs"][:R], B["yfull"][:T], B["rs"][:T]
        qkv, q, att, ors, gu, act = B["qkv"][:T], B["q"][:T], B["att"][:T], B["ors"][:T], B["gu"][:T], B["act"][:T]
        if T != T0:
            att[T0:].zero_()
        S = meta.sample_rows
        chk = self.checked and S is not None and S.numel() > 0
        S_loc = torch.remainder(S, R).to(torch.int32) if chk else None
        torch.index_select(self.embed, 0, meta.tokens[self.rank * R:(self.rank + 1) * R], out=xs)
        for i, lw in enumerate(self.layers):
            lc = cache[i]
            ys = self._norm_into_shard(xs, lw.ln1, None if i == 0 else B["resid"][:R], R)
            if chk:
                self._norm_replay(ys, lw.ln1, R, S_loc, f"L{i}.norm1")
            yrs = self._gather_rows(ys, R, yfull, rs)
            self._linear(yfull, lw.qkv, lw.cw.get("qkv"), f"L{i}.qkv", qkv, yrs, sample=S)
            layers.qk_norm_rope_kv(qkv, nq, nkv, meta.pos, meta.slots, lw.q_norm, lw.k_norm, cfg.rms_eps, self.rope,
                                   q, lc)
            if chk:
                layers.qk_norm_rope_kv(qkv, nq, nkv, meta.pos, meta.slots, lw.q_norm, lw.k_norm, cfg.rms_eps,
                                       self.rope, q, lc, rows=S, check=self._st(f"L{i}.rope_kv"))
            if self.checked:
                ors.zero_()
            if meta.mode == "prefill":
                attention.prefill(q, lc, meta.block_table, meta.pos, meta.tiles, nq, nkv, out=att,
                                  row_sq=ors if self.checked else None)
                if chk:
                    attention.prefill(q, lc, meta.block_table, meta.pos, meta.sample_tiles, nq, nkv, out=att,
                                      row_idx=meta.sample_idx, check=self._st(f"L{i}.attn"))
            else:
                scratch = self.decode_scratch(T0, meta.max_ctx)
                attention.decode(q[:T0], lc, meta.block_table, meta.seq_req, meta.ctx, nq, nkv, meta.max_ctx,
                                 out=att[:T0], row_sq=ors if self.checked else None, scratch=scratch)
                if chk:
                    attention.decode(q[:T0], lc, meta.block_table, meta.seq_req, meta.ctx, nq, nkv, meta.max_ctx,
                                     out=att[:T0], seq_idx=S, scratch=scratch, check=self._st(f"L{i}.attn"))
            self._rowpar(att.view(T, nq * D), lw.o, lw.cw.get("o"), f"L{i}.o", T, R, ors, xs, sample=S)
            ys = self._norm_into_shard(xs, lw.ln2, B["resid"][:R], R)
            if chk:
                self._norm_replay(ys, lw.ln2, R, S_loc, f"L{i}.norm2")
            yrs = self._gather_rows(ys, R, yfull, rs)
            self._linear(yfull, lw.gate_up, lw.cw.get("gate_up"), f"L{i}.gate_up", gu, yrs, sample=S)
            layers.silu_mul(gu, out=act, row_sq=rs)
            if chk:
                layers.silu_mul(gu, out=act, rows=S, check=self._st(f"L{i}.act"))
            self._rowpar(act, lw.down, lw.cw.get("down"), f"L{i}.down", T, R, rs, xs, sample=S)
        ys = self._norm_into_shard(xs, self.final_ln, B["resid"][:R], R)
        if chk:
            self._norm_replay(ys, self.final_ln, R, S_loc, "final_norm")
        self._ag(ys, R, yfull)
        yl = yfull.index_select(0, meta.logits_rows)
        logits = torch.empty(yl.shape[0], self.vocab_l, dtype=torch.bfloat16, device=dev)
        if self.checked:
            gemm.checked_linear(yl, self.lm_cw, self.state.state, self.slot["lm_head"], out=logits)
        else:
            torch.matmul(yl, self.lm_head.t(), out=logits)
        return logits

    def sample(self, logits: torch.Tensor) -> torch.Tensor:
        """Greedy token over the vocabulary shards of all ranks."""
        if self.world == 1:
            return torch.argmax(logits, dim=-1)
        mx, idx = logits.float().max(dim=-1)
        pair = torch.stack([mx, (idx + self.rank * self.vocab_l).float()], dim=-1)     # (L, 2)
        allp = torch.empty(self.world, *pair.shape, dtype=pair.dtype, device=pair.device)
        dist.all_gather_into_tensor(allp, pair)
        best = allp[..., 0].argmax(dim=0)                                              # (L,)
        return allp[..., 1].gather(0, best.view(1, -1)).view(-1).long()
