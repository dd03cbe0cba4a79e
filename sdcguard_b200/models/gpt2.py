"""GPT-2 (small: 12 layers, d=768, 12 heads, vocab 50257, context 1024) in plain PyTorch, random-init N(0, 0.02):
the CPU fp32 benchmark model. Every projection is an nn.Linear (c_attn, c_proj, c_fc, mlp c_proj, lm_head), so
`numerics.cpu_abft.protect_cpu` checks all 49 of them; the LM head shares the token embedding weight.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass(frozen=True)
class GPT2Config:
    layers: int = 12
    hidden: int = 768
    heads: int = 12
    vocab: int = 50257
    context: int = 1024


class Block(nn.Module):
    def __init__(self, c: GPT2Config):
        super().__init__()
        self.heads = c.heads
        self.ln_1 = nn.LayerNorm(c.hidden)
        self.c_attn = nn.Linear(c.hidden, 3 * c.hidden)
        self.attn_proj = nn.Linear(c.hidden, c.hidden)
        self.ln_2 = nn.LayerNorm(c.hidden)
        self.c_fc = nn.Linear(c.hidden, 4 * c.hidden)
        self.mlp_proj = nn.Linear(4 * c.hidden, c.hidden)

    def forward(self, x):
        B, T, H = x.shape
        q, k, v = self.c_attn(self.ln_1(x)).split(H, dim=-1)
        sh = (B, T, self.heads, H // self.heads)
        q, k, v = (t.view(sh).transpose(1, 2) for t in (q, k, v))
        a = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        x = x + self.attn_proj(a.transpose(1, 2).reshape(B, T, H))
        return x + self.mlp_proj(F.gelu(self.c_fc(self.ln_2(x)), approximate="tanh"))


class GPT2(nn.Module):
    def __init__(self, c: GPT2Config = GPT2Config(), seed: int = 0):
        super().__init__()
        self.c = c
        self.wte = nn.Embedding(c.vocab, c.hidden)
        self.wpe = nn.Embedding(c.context, c.hidden)
        self.h = nn.ModuleList(Block(c) for _ in range(c.layers))
        self.ln_f = nn.LayerNorm(c.hidden)
        self.lm_head = nn.Linear(c.hidden, c.vocab, bias=False)
        g = torch.Generator().manual_seed(seed)
        with torch.no_grad():
            for n, p in self.named_parameters():
                if p.dim() >= 2:
                    p.normal_(0.0, 0.02, generator=g)
                elif n.endswith("bias"):
                    p.zero_()
            for blk in self.h:               # GPT-2's scaled init of the residual projections
                for lin in (blk.attn_proj, blk.mlp_proj):
                    lin.weight.mul_(1.0 / math.sqrt(2 * c.layers))
        self.lm_head.weight = self.wte.weight

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        T = ids.shape[1]
        x = self.wte(ids) + self.wpe(torch.arange(T, device=ids.device))
        for blk in self.h:
            x = blk(x)
        return self.lm_head(self.ln_f(x))
