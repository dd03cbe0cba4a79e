"""Mixture-of-experts layer (Mixtral-style: softmax router, top-k, renormalised weights, SwiGLU experts) on this
library's kernels, expert-parallel over the ranks:

    logits = checked GEMM  x @ Wr^T                 ABFT (router rows padded to a multiple of 8)
    ids, w = router_topk(logits)                     exact replay of a rotating sample of tokens
    rows   = dispatch(x, ids)                        sealed transfer over NVLink, verified on arrival
    per local expert e:  h = silu(x_e Wg^T) * (x_e Wu^T);  y_e = h Wd^T      ABFT on both GEMMs
    y      = combine(y_e, w)                         sealed transfer back, verified, weighted sum in fp32

Expert weights are generated per global expert from a seed, so every rank can build the same reference and any
EP size builds the same model. Config: Mixtral-8x7B shape = hidden 4096, 8 experts, top-2, expert FFN 14336.

Reference: the reference samples rows of vLLM's fused MoE for recompute (src/sdcguard/serve_moe.py:123-165,
`MoEChecks` :748) and the router for replay (src/sdcguard/serve_route.py, `RouteChecks` :588); it does not check
the expert-parallel all-to-all.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from ..ops import gemm, layers
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
                 collective: str = "own"):
        """collective "own": the sealed peer-memory all-to-all (needs comm); "nccl": the unchecked baseline
        exchange over torch.distributed (comm may be None)."""
        self.H, self.I, self.E, self.k = hidden, inter, experts, top_k
        self.comm = comm
        self.collective = collective
        self.device = torch.device(device)
        self.checked = checked
        if comm is not None:
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
            self.cw13 = [gemm.CheckedWeight(w) for w in self.w13]
            self.cw2 = [gemm.CheckedWeight(w) for w in self.w2]
        self.attach(state or gemm.StateTable(self.device, 8 + 2 * self.epr), name)

    def attach(self, table: gemm.StateTable, name: str) -> None:
        """Register this layer's check slots in `table` (a model's shared state table)."""
        self.state = table
        self.name = name
        self.slots = {}
        if not self.checked:
            return
        self.slots["router"] = table.add(f"{name}.router (ABFT GEMM)", self.cw_r.nb)
        self.slots["route"] = table.add(f"{name}.route (replay)", 1)
        for j, e in enumerate(self.local):
            self.slots[f"up{j}"] = table.add(f"{name}.expert{e}.gate_up (ABFT GEMM)", self.cw13[j].nb)
            self.slots[f"down{j}"] = table.add(f"{name}.expert{e}.down (ABFT GEMM)", self.cw2[j].nb)

    def inject_next(self, slot: str, row: int, col: int, bit: int) -> None:
        """Fault injection: flip `bit` of fp32 accumulator (row, col) of the next GEMM in `slot` ("router",
        "up<j>" or "down<j>" for local expert j) before its check."""
        self._inject = (slot, (row, col, 1 << bit))

    def _lin(self, x, w, cw, slot, out=None):
        if not self.checked:
            return torch.matmul(x, w.t(), out=out) if out is not None else torch.matmul(x, w.t())
        inj = None
        if getattr(self, "_inject", None) and self._inject[0] == slot:
            inj, self._inject = self._inject[1], None
        return gemm.checked_linear(x, cw, self.state.state, self.slots[slot], out=out, inject=inj)

    def forward(self, x: torch.Tensor, sample: Optional[torch.Tensor] = None) -> torch.Tensor:
        logits = self._lin(x, self.router, getattr(self, "cw_r", None), "router")
        ids, wts = router_topk(logits[:, : self.E], self.k)
        if self.checked and sample is not None and sample.numel():
            router_topk(logits[:, : self.E], self.k, ids, wts, rows=sample, check=self.state.state[self.slots["route"]])
        self.last_ids, self.last_wts = ids, wts
        if self.collective == "nccl":
            return self._forward_nccl(x, ids, wts)
        xe, offs = self.comm.dispatch(x, ids)
        ye = torch.empty_like(xe)
        self._experts(xe, offs, ye)
        return self.comm.combine(ye, wts)

    def _experts(self, xe, offs, ye):
        for j in range(self.epr):
            a, b = offs[j], offs[j + 1]
            if b == a:
                continue
            h = self._lin(xe[a:b], self.w13[j], getattr(self, "cw13", [None] * self.epr)[j], f"up{j}")
            act, _ = layers.silu_mul(h)
            self._lin(act, self.w2[j], getattr(self, "cw2", [None] * self.epr)[j], f"down{j}", out=ye[a:b])

    def _forward_nccl(self, x, ids, wts):
        """Baseline exchange: all_to_all_single of rows sorted by expert, cuBLAS experts, all_to_all back."""
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
        sc = cnt_e.view(self.world, self.epr).sum(1).tolist()
        rc_m = recv_cnt.view(self.world, self.epr).tolist()
        rc = [sum(r) for r in rc_m]
        recv = torch.empty(sum(rc), self.H, dtype=x.dtype, device=x.device)
        if self.world > 1:
            dist.all_to_all_single(recv, send, rc, sc)
        else:
            recv.copy_(send)
        # received rows: by source, then local expert; regroup by expert for the GEMMs
        starts, pos = [], 0
        for src in range(self.world):
            for e in range(self.epr):
                starts.append((e, src, pos, rc_m[src][e]))
                pos += rc_m[src][e]
        perm = [i for e in range(self.epr) for (ee, src, p0, n) in starts if ee == e for i in range(p0, p0 + n)]
        perm_t = torch.tensor(perm, dtype=torch.long, device=x.device)
        xe = recv.index_select(0, perm_t)
        offs = [0]
        for e in range(self.epr):
            offs.append(offs[-1] + sum(rc_m[src][e] for src in range(self.world)))
        ye = torch.empty_like(xe)
        self._experts(xe, offs, ye)
        back = torch.empty_like(recv)
        back.index_copy_(0, perm_t, ye)
        ret = torch.empty_like(send)
        if self.world > 1:
            dist.all_to_all_single(ret, back, sc, rc)
        else:
            ret.copy_(back)
        y = torch.zeros(T, self.H, dtype=torch.float32, device=x.device)
        y.index_add_(0, order // K, ret.float() * wts.view(-1)[order].unsqueeze(1))
        return y.to(torch.bfloat16)


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
