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
    def __init__(self, hidden: int, inter: int, experts: int, top_k: int, comm: EPComm, device, checked: bool = True,
                 seed: int = 0, state: Optional[gemm.StateTable] = None, name: str = "moe"):
        self.H, self.I, self.E, self.k = hidden, inter, experts, top_k
        self.comm = comm
        self.device = torch.device(device)
        self.checked = checked
        self.rank, self.world = comm.rank, comm.world
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
        self.state = state or gemm.StateTable(self.device, 8 + 2 * self.epr)
        self.slots = {}
        if checked:
            self.cw_r = gemm.CheckedWeight(self.router)
            self.slots["router"] = self.state.add(f"{name}.router (ABFT GEMM)", self.cw_r.nb)
            self.slots["route"] = self.state.add(f"{name}.route (replay)", 1)
            self.cw13 = [gemm.CheckedWeight(w) for w in self.w13]
            self.cw2 = [gemm.CheckedWeight(w) for w in self.w2]
            for j, e in enumerate(self.local):
                self.slots[f"up{j}"] = self.state.add(f"{name}.expert{e}.gate_up (ABFT GEMM)", self.cw13[j].nb)
                self.slots[f"down{j}"] = self.state.add(f"{name}.expert{e}.down (ABFT GEMM)", self.cw2[j].nb)

    def _lin(self, x, w, cw, slot, out=None):
        if not self.checked:
            return torch.matmul(x, w.t(), out=out) if out is not None else torch.matmul(x, w.t())
        return gemm.checked_linear(x, cw, self.state.state, self.slots[slot], out=out)

    def forward(self, x: torch.Tensor, sample: Optional[torch.Tensor] = None) -> torch.Tensor:
        logits = self._lin(x, self.router, getattr(self, "cw_r", None), "router")
        ids, wts = router_topk(logits[:, : self.E], self.k)
        if self.checked and sample is not None and sample.numel():
            router_topk(logits[:, : self.E], self.k, ids, wts, rows=sample, check=self.state.state[self.slots["route"]])
        self.last_ids, self.last_wts = ids, wts
        xe, offs = self.comm.dispatch(x, ids)
        ye = torch.empty_like(xe)
        for j in range(self.epr):
            a, b = offs[j], offs[j + 1]
            if b == a:
                continue
            h = self._lin(xe[a:b], self.w13[j], getattr(self, "cw13", [None] * self.epr)[j], f"up{j}")
            act, _ = layers.silu_mul(h)
            self._lin(act, self.w2[j], getattr(self, "cw2", [None] * self.epr)[j], f"down{j}", out=ye[a:b])
        return self.comm.combine(ye, wts)


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
