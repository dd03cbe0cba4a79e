"""Mixture-of-experts layer (Mixtral-style: softmax router, top-k, renormalised weights, SwiGLU experts) on this
library's kernels, expert-parallel over the ranks or with every expert on this GPU:

    logits = checked GEMM  x @ Wr^T                 ABFT (router rows padded to a multiple of 8)
    ids, w = router_topk(logits)                     exact replay of a rotating sample of tokens
    rows   = dispatch(x, ids)                        "own": sealed transfer over NVLink, verified on arrival;
                                                     "local": on-device grouping (ops.moe.Grouping)
    h      = grouped checked GEMM  rows @ W13_e^T    ABFT, all local experts in one launch (rows of each expert
    a      = silu(h_gate) * h_up                     start on a 128-row band; band -> expert table on the device)
    y_e    = grouped checked GEMM  a @ W2_e^T        ABFT, one launch
    (precision "fp8": before each expert GEMM the grouped rows are quantized to E4M3 with 1 x 128 power-of-two
    scales, a rotating sample of rows replayed exactly; the expert GEMMs are the grouped block-scaled fp8 checked
    GEMM on 128 x 128-scaled E4M3 expert weights)
    y      = combine(y_e, w)                         sealed transfer back ("own"), weighted sum in fp32, k order

Nothing in a checked layer reads back to the host: the band table and band count the grouped GEMMs need are written
by the dispatch (or grouping) kernel, so a step of MoE layers can be captured in a CUDA graph. The "nccl" arm is the
unchecked baseline: torch.distributed all-to-all and PyTorch's grouped GEMM.

Expert weights are generated per global expert from a seed, so every rank can build the same reference and any
EP size builds the same model. Config: Mixtral-8x7B shape = hidden 4096, 8 experts, top-2, expert FFN 14336.

Reference: the reference samples rows of vLLM's fused MoE for recompute (src/sdcguard/serve_moe.py:123-165,
`MoEChecks` :748), checks PyTorch's `_grouped_mm` per group (src/sdcguard/guard.py:102-143) and replays the router
(src/sdcguard/serve_route.py, `RouteChecks` :588); it does not check the expert-parallel all-to-all.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from ..ops import gemm, layers
from ..ops import moe as moe_ops
from ..parallel.ep import EPComm, router_topk


def expert_weights(seed: int, e: int, hidden: int, inter: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    g = torch.Generator(device=device).manual_seed(seed * 7919 + 104729 * (e + 1))
    w13 = torch.empty(2 * inter, hidden, device=device).normal_(0.0, 0.02, generator=g).to(torch.bfloat16)
    w2 = torch.empty(hidden, inter, device=device).normal_(0.0, 0.02, generator=g).to(torch.bfloat16)
    return w13, w2


def router_weight(seed: int, experts: int, hidden: int, device) -> torch.Tensor:
    g = torch.Generator(device=device).manual_seed(seed * 7919 + 17)
    return torch.empty(experts, hidden, device=device).normal_(0.0, 1.0 / hidden ** 0.5, generator=g).to(torch.bfloat16)


class MoELayer:
    def __init__(self, hidden: int, inter: int, experts: int, top_k: int, comm: Optional[EPComm], device,
                 checked: bool = True, seed: int = 0, state: Optional[gemm.StateTable] = None, name: str = "moe",
                 collective: str = "own", precision: str = "bf16"):
        """collective "own": the sealed peer-memory all-to-all (needs comm); "local": every expert on this GPU,
        rows grouped on the device (no all-to-all, comm unused); "nccl": the unchecked baseline exchange over
        torch.distributed (comm may be None). precision "fp8" (checked only): block-scaled fp8 expert GEMMs."""
        if collective not in ("own", "local", "nccl"):
            raise ValueError(f"collective {collective!r}: own, local or nccl")
        if precision not in ("bf16", "fp8") or (precision == "fp8" and not checked):
            raise ValueError("precision must be bf16, or fp8 with checked=True")
        self.precision = precision
        self.H, self.I, self.E, self.k = hidden, inter, experts, top_k
        self.comm = comm
        self.collective = collective
        self.device = torch.device(device)
        self.checked = checked
        if collective == "local":
            self.rank, self.world = 0, 1
        elif comm is not None:
            self.rank, self.world = comm.rank, comm.world
        else:
            self.rank = dist.get_rank() if dist.is_initialized() else 0
            self.world = dist.get_world_size() if dist.is_initialized() else 1
        self.epr = experts // self.world
        self.local = list(range(self.rank * self.epr, (self.rank + 1) * self.epr))
        rw = router_weight(seed, experts, hidden, self.device)
        self.er = -(-experts // 8) * 8
        self.router = torch.zeros(self.er, hidden, dtype=torch.bfloat16, device=self.device)
        self.router[:experts] = rw
        self.w13, self.w2 = [], []
        for e in self.local:
            a, b = expert_weights(seed, e, hidden, inter, self.device)
            self.w13.append(a)
            self.w2.append(b)
        self.name = name
        if checked:
            self.cw_r = gemm.CheckedWeight(self.router)
        if checked and precision == "fp8":
            from ..ops import fp8 as fp8_ops
            self.f13 = fp8_ops.Fp8WeightStack(self.w13)
            self.f2 = fp8_ops.Fp8WeightStack(self.w2)
            self._qturn = 0
        elif checked:
            self.s13 = gemm.CheckedWeightStack(self.w13)
            self.s2 = gemm.CheckedWeightStack(self.w2)
            # the per-expert weights become views of the stacks (one copy of the expert weights in memory)
            self.w13 = [self.s13.expert(j) for j in range(self.epr)]
            self.w2 = [self.s2.expert(j) for j in range(self.epr)]
        self._grouping: Optional[moe_ops.Grouping] = None
        self._bufs: dict = {}
        self.baseline_path = None
        self.attach(state or gemm.StateTable(self.device, 8), name)

    def attach(self, table: gemm.StateTable, name: str) -> None:
        """Register this layer's check slots in `table` (a model's shared state table)."""
        self.state = table
        self.name = name
        self.slots = {}
        if not self.checked:
            return
        self.slots["router"] = table.add(f"{name}.router (ABFT GEMM)", self.cw_r.nb)
        self.slots["route"] = table.add(f"{name}.route (replay)", 1)
        if self.precision == "fp8":
            self.slots["up"] = table.add(f"{name}.experts.gate_up (ABFT fp8 GEMM)", self.f13.nb)
            self.slots["down"] = table.add(f"{name}.experts.down (ABFT fp8 GEMM)", self.f2.nb)
            self.slots["up.q"] = table.add(f"{name}.experts.gate_up.quant (replay)", 1)
            self.slots["down.q"] = table.add(f"{name}.experts.down.quant (replay)", 1)
            return
        self.slots["up"] = table.add(f"{name}.experts.gate_up (ABFT GEMM)", self.s13.nb)
        self.slots["down"] = table.add(f"{name}.experts.down (ABFT GEMM)", self.s2.nb)

    def inject_next(self, slot: str, row: int, col: int, bit: int) -> None:
        """Fault injection: flip `bit` of fp32 accumulator (row, col) of the next GEMM in `slot` before its check:
        "router" (row = token), "up" or "down" (row = row of the grouped expert input: the experts' rows on 128-row
        bands in local expert order)."""
        self._inject = (slot, (row, col, 1 << bit))

    def _take(self, slot):
        if getattr(self, "_inject", None) and self._inject[0] == slot:
            inj, self._inject = self._inject[1], None
            return inj
        return None

    def _lin(self, x, w, cw, slot, out=None):
        if not self.checked:
            return torch.matmul(x, w.t(), out=out) if out is not None else torch.matmul(x, w.t())
        return gemm.checked_linear(x, cw, self.state.state, self.slots[slot], out=out, inject=self._take(slot))

    def forward(self, x: torch.Tensor, sample: Optional[torch.Tensor] = None) -> torch.Tensor:
        logits = self._lin(x, self.router, getattr(self, "cw_r", None), "router")
        ids, wts = router_topk(logits[:, : self.E], self.k)
        if self.checked and sample is not None and sample.numel():
            router_topk(logits[:, : self.E], self.k, ids, wts, rows=sample, check=self.state.state[self.slots["route"]])
        self.last_ids, self.last_wts = ids, wts
        if self.collective == "nccl":
            return self._forward_nccl(x, ids, wts)
        if not self.checked:
            raise ValueError("the unchecked arm uses collective 'nccl'")
        if self.collective == "local":
            grp = self._grouping_for(x.shape[0])
            xg, rsq = grp.group(x, ids)
            yg = self._experts_grouped(xg, rsq, grp.gband, grp.gcount, x.shape[0] * self.k)
            return grp.combine(yg, wts)
        xg, rsq, gband, gcount = self.comm.dispatch_grouped(x, ids)
        yg = self._experts_grouped(xg, rsq, gband, gcount, x.shape[0] * self.k // max(1, self.world))
        return self.comm.combine(yg, wts)

    def _grouping_for(self, T: int) -> moe_ops.Grouping:
        g = self._grouping
        if g is None or g.T < T:
            g = self._grouping = moe_ops.Grouping(max(T, 1), self.k, self.epr, self.H, self.device, e_lo=self.local[0])
        return g

    def _buffers(self, cap: int):
        b = self._bufs
        if b.get("cap", 0) < cap:
            dev, bf = self.device, torch.bfloat16
            b.update(cap=cap, h=torch.empty(cap, 2 * self.I, dtype=bf, device=dev),
                     act=torch.empty(cap, self.I, dtype=bf, device=dev),
                     act_sq=torch.empty(cap, dtype=torch.float32, device=dev),
                     y=torch.empty(cap, self.H, dtype=bf, device=dev))
            if self.precision == "fp8":
                from ..ops import fp8 as fp8_ops
                b.update(qx=_fp8_act(fp8_ops, cap, self.H, dev), qa=_fp8_act(fp8_ops, cap, self.I, dev))
        return b

    def _quant_sample(self, rows_valid: int) -> torch.Tensor:
        """A rotating sample of grouped rows to replay the quantization of: rows below T k lie in bands in use."""
        n = max(1, min(8, rows_valid))
        self._qturn += 1
        r = (torch.arange(n, dtype=torch.int64) * 131 + self._qturn * 8) % max(1, rows_valid)
        return r.to(torch.int32).to(self.device, non_blocking=True)

    def _experts_grouped(self, xg, rsq, gband, gcount, rows_valid: int = 0):
        """Both expert GEMMs of every local expert as two grouped checked launches (and SwiGLU between)."""
        cap = xg.shape[0]
        b = self._buffers(cap)
        st = self.state.state
        if self.precision == "fp8":
            return self._experts_grouped_fp8(xg, gband, gcount, rows_valid, b, st)
        h = gemm.checked_linear_grouped(xg, self.s13, gband, gcount, st, self.slots["up"], row_sq=rsq,
                                        out=b["h"][:cap], inject=self._take("up"))
        act, asq = layers.silu_mul_bands(h, gcount, out=b["act"][:cap], row_sq=b["act_sq"][:cap])
        return gemm.checked_linear_grouped(act, self.s2, gband, gcount, st, self.slots["down"], row_sq=asq,
                                           out=b["y"][:cap], inject=self._take("down"))

    def _experts_grouped_fp8(self, xg, gband, gcount, rows_valid, b, st):
        from ..ops import fp8 as fp8_ops
        cap = xg.shape[0]
        qx = fp8_ops.quantize_act(xg, out=_fp8_view(b["qx"], cap))
        if rows_valid > 0:
            fp8_ops.quantize_act(xg, out=qx, rows=self._quant_sample(rows_valid), check=st[self.slots["up.q"]])
        h = fp8_ops.checked_linear_fp8_grouped(qx, self.f13, gband, gcount, st, self.slots["up"], out=b["h"][:cap],
                                               inject=self._take("up"))
        act, _ = layers.silu_mul_bands(h, gcount, out=b["act"][:cap], row_sq=b["act_sq"][:cap])
        qa = fp8_ops.quantize_act(act, out=_fp8_view(b["qa"], cap))
        if rows_valid > 0:
            fp8_ops.quantize_act(act, out=qa, rows=self._quant_sample(rows_valid), check=st[self.slots["down.q"]])
        return fp8_ops.checked_linear_fp8_grouped(qa, self.f2, gband, gcount, st, self.slots["down"],
                                                  out=b["y"][:cap], inject=self._take("down"))

    def _experts_unchecked(self, xe, offs_host):
        """Baseline expert MLPs: PyTorch's grouped GEMM when it runs here, else one cuBLAS GEMM per expert."""
        if self.baseline_path in (None, "grouped_mm") and hasattr(torch, "_grouped_mm") and xe.shape[0] > 0:
            try:
                if "w13_t" not in self._bufs:
                    self._bufs["w13_t"] = torch.stack(self.w13).transpose(1, 2)     # (E, H, 2I), column-major
                    self._bufs["w2_t"] = torch.stack(self.w2).transpose(1, 2)       # (E, I, H)
                ends = torch.tensor(offs_host[1:], dtype=torch.int32, device=xe.device)
                h = torch._grouped_mm(xe, self._bufs["w13_t"], offs=ends)
                act, _ = layers.silu_mul(h)
                y = torch._grouped_mm(act, self._bufs["w2_t"], offs=ends)
                self.baseline_path = "grouped_mm"
                return y
            except (RuntimeError, TypeError, NotImplementedError):
                self.baseline_path = "per_expert"
        self.baseline_path = "per_expert"
        ye = torch.empty_like(xe)
        for j in range(self.epr):
            a, b = offs_host[j], offs_host[j + 1]
            if b > a:
                h = torch.matmul(xe[a:b], self.w13[j].t())
                act, _ = layers.silu_mul(h)
                torch.matmul(act, self.w2[j].t(), out=ye[a:b])
        return ye

    def _forward_nccl(self, x, ids, wts):
        """Baseline exchange: all_to_all_single of rows sorted by expert, unchecked experts, all_to_all back. The
        split sizes are read to the host once per layer (all_to_all_single takes host lists); every permutation
        is built on the device."""
        T, K = ids.shape
        flat = ids.view(-1).long()
        order = torch.argsort(flat, stable=True)
        send = x.index_select(0, order // K)
        cnt_e = torch.bincount(flat, minlength=self.E).to(torch.int64)          # rows per global expert
        recv_cnt = torch.empty_like(cnt_e)
        if self.world > 1:
            dist.all_to_all_single(recv_cnt, cnt_e)                               # (src, local expert) counts
        else:
            recv_cnt.copy_(cnt_e)
        both = torch.stack([cnt_e, recv_cnt]).cpu()
        sc = both[0].view(self.world, self.epr).sum(1).tolist()
        rc_m = both[1].view(self.world, self.epr)
        rc = rc_m.sum(1).tolist()
        recv = torch.empty(sum(rc), self.H, dtype=x.dtype, device=x.device)
        if self.world > 1:
            dist.all_to_all_single(recv, send, rc, sc)
        else:
            recv.copy_(send)
        # received rows come by source, then local expert: regroup by expert with a stable sort of expert ids
        dev = x.device
        eid = torch.repeat_interleave(torch.arange(self.epr, device=dev).repeat(self.world),
                                      rc_m.reshape(-1).to(dev))
        perm = torch.argsort(eid, stable=True)
        xe = recv.index_select(0, perm)
        per_e = rc_m.sum(0).tolist()
        offs = [0]
        for n in per_e:
            offs.append(offs[-1] + n)
        ye = self._experts_unchecked(xe, offs)
        back = torch.empty_like(recv)
        back.index_copy_(0, perm, ye)
        ret = torch.empty_like(send)
        if self.world > 1:
            dist.all_to_all_single(ret, back, sc, rc)
        else:
            ret.copy_(back)
        y = torch.zeros(T, self.H, dtype=torch.float32, device=dev)
        y.index_add_(0, order // K, ret.float() * wts.view(-1)[order].unsqueeze(1))
        return y.to(torch.bfloat16)


def _fp8_act(fp8_ops, cap: int, k: int, dev):
    return fp8_ops.Fp8Act(torch.empty(cap, k, dtype=torch.float8_e4m3fn, device=dev),
                          torch.empty(cap, k // 128, dtype=torch.float32, device=dev),
                          torch.empty(cap, dtype=torch.float32, device=dev),
                          torch.full((-(-cap // 128), k // 128, 512), 127, dtype=torch.uint8, device=dev))


def _fp8_view(a, rows: int):
    """The first `rows` rows of an activation buffer (scale-factor chunks by whole 128-row tiles)."""
    return type(a)(a.q[:rows], a.sa[:rows], a.row_sq[:rows], a.sf[: -(-rows // 128)])


def reference_moe(x: torch.Tensor, seed: int, hidden: int, inter: int, experts: int, top_k: int,
                  ids: Optional[torch.Tensor] = None, w: Optional[torch.Tensor] = None):
    """fp32 PyTorch reference of the layer (all experts on this device). With ids / w given, uses that routing
    (the router is compared separately: bf16 logits can tie)."""
    dev = x.device
    if ids is None:
        rw = router_weight(seed, experts, hidden, dev).float()
        logits = (x.float() @ rw.t()).to(torch.bfloat16).float()
        p = torch.softmax(logits, dim=-1)
        w, ids = torch.topk(p, top_k, dim=-1)
        w = w / w.sum(-1, keepdim=True)
    ids, w = ids.long(), w.float()
    out = torch.zeros(x.shape[0], hidden, device=dev)
    for e in range(experts):
        w13, w2 = expert_weights(seed, e, hidden, inter, dev)
        sel = (ids == e)
        rows = sel.any(-1).nonzero().view(-1)
        if rows.numel() == 0:
            continue
        h = x[rows].float() @ w13.float().t()
        g, u = h[:, :inter], h[:, inter:]
        a = (torch.nn.functional.silu(g) * u).to(torch.bfloat16).float()
        y = a @ w2.float().t()
        wk = (w * sel.float()).sum(-1)[rows]
        out[rows] += wk[:, None] * y
    return out, ids
