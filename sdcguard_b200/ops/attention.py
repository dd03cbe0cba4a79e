"""Paged attention entry points (`csrc/attention.cu`): causal prefill over a batch of requests and single-token
decode, both over a paged KV cache with 16-token pages, plus the host-side tiling of prefill work.

Rows of both kernels are deterministic (see the kernel file), so `replay_*` recompute a sample of rows on
separate CTAs and `ops.layers.compare_rows` checks them bit for bit. The reference samples (token, head) pairs
and recomputes them in fp32 against an error bound (src/sdcguard/serve_attn.py:5-48, `attn_check_triton`
:574); the replay needs no bound, so every flipped bit in a sampled row is seen.
"""
from __future__ import annotations

import math
from typing import Optional, Sequence

import torch

from .. import _native

ROWS = 128


def _s(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _pairs(per_request: list[list[tuple]]) -> list[tuple]:
    """Tiles two by two within each request (the prefill kernel runs the two tiles of a pair in one CTA on shared
    key / value tiles); a request with an odd number of tiles gets an empty partner (0 tokens)."""
    pairs = []
    for tiles in per_request:
        for i in range(0, len(tiles), 2):
            a = tiles[i]
            b = tiles[i + 1] if i + 1 < len(tiles) else (a[0], a[1] + a[2], 0, -1)
            pairs.append((a, b))
    return pairs


def prefill_tiles(q_starts: Sequence[int], q_lens: Sequence[int], group: int) -> torch.Tensor:
    """(2 n, 4) int32 tiles (request, first token, tokens, -1) covering every request's new tokens, as n pairs of
    consecutive tiles of one request (entries 2i and 2i + 1), pairs ordered by the keys they attend to, most first
    (later tiles of a causal prompt attend to more keys), so the longest CTAs start first."""
    tpc = ROWS // group
    per = [[(r, s + off, min(tpc, n - off), -1) for off in range(0, n, tpc)] for r, (s, n) in
           enumerate(zip(q_starts, q_lens))]
    pairs = _pairs(per)
    # keys a pair attends to: its last token's position within its request
    pairs.sort(key=lambda pr: -(pr[0][1] - q_starts[pr[0][0]] + pr[0][2] + pr[1][2]))
    flat = [t for pr in pairs for t in pr]
    return torch.tensor(flat, dtype=torch.int32).view(-1, 4)


def replay_tiles(sampled: Sequence[Sequence[int]], group: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Tiles for a replay of sampled tokens (sampled[r] lists request r's sampled token indices), in pairs of one
    request as `prefill_tiles` makes them; returns (tiles, row_idx)."""
    tpc = ROWS // group
    per, idx = [], []
    for r, toks in enumerate(sampled):
        mine = []
        for off in range(0, len(toks), tpc):
            chunk = list(toks[off:off + tpc])
            mine.append((r, 0, len(chunk), len(idx)))
            idx.extend(chunk)
        per.append(mine)
    flat = [t for pr in _pairs(per) for t in pr]
    t = torch.tensor(flat, dtype=torch.int32).view(-1, 4)
    return t, torch.tensor(idx, dtype=torch.int32)


def prefill(q: torch.Tensor, cache: torch.Tensor, block_table: torch.Tensor, pos: torch.Tensor,
            tiles: torch.Tensor, nq: int, nkv: int, out: Optional[torch.Tensor] = None,
            row_idx: Optional[torch.Tensor] = None, row_sq: Optional[torch.Tensor] = None,
            scale: Optional[float] = None, check: Optional[torch.Tensor] = None) -> torch.Tensor:
    """q: (T, nq, 128) bf16; tiles/row_idx/pos/block_table int32 on the device. out: (T, nq, 128) or, for a
    replay, any tensor indexed by the same token ids. With `check` (a state row; replay tiles and row_idx
    given), the sampled rows are recomputed and compared with `out` instead of written."""
    if out is None:
        out = torch.empty_like(q)
    scale = 1.0 / math.sqrt(128) if scale is None else scale
    _native.check(_native.lib().sdc_attn_prefill(
        q.data_ptr(), out.data_ptr(), cache.data_ptr(), cache.shape[0], block_table.data_ptr(), block_table.shape[1],
        pos.data_ptr(), tiles.data_ptr(), tiles.shape[0], None if row_idx is None else row_idx.data_ptr(), nq, nkv,
        128, float(scale), None if row_sq is None else row_sq.data_ptr(), None if check is None else check.data_ptr(),
        _s(q)), "attention prefill")
    return out


def decode_scratch(nseq_rows: int, nq: int, nkv: int, max_ctx: int, device) -> torch.Tensor:
    """Partial-result scratch for `decode` (one record per sequence, kv head and 256-key segment)."""
    splits = int(_native.lib().sdc_attn_decode_splits(int(max_ctx)))
    return torch.empty(nseq_rows * nkv * splits * (nq // nkv) * 132, dtype=torch.float32, device=device)


def decode(q: torch.Tensor, cache: torch.Tensor, block_table: torch.Tensor, seq_req: torch.Tensor,
           ctx: torch.Tensor, nq: int, nkv: int, max_ctx: int, out: Optional[torch.Tensor] = None,
           seq_idx: Optional[torch.Tensor] = None, nseq: Optional[int] = None,
           row_sq: Optional[torch.Tensor] = None, scale: Optional[float] = None,
           scratch: Optional[torch.Tensor] = None, check: Optional[torch.Tensor] = None) -> torch.Tensor:
    """q: (B, nq, 128); split-KV: a CTA per (sequence, kv head) and every z-th 256-key segment (64-key chunks merged
    in order inside the segment), then a fixed-order combine of the segments.
    seq_idx selects sequences to run (replay). scratch: from `decode_scratch` (allocated here if absent).
    With `check` (a state row; seq_idx given), the selected rows are recomputed and compared with `out`."""
    if out is None:
        out = torch.empty_like(q)
    scale = 1.0 / math.sqrt(128) if scale is None else scale
    n = nseq if nseq is not None else (seq_idx.shape[0] if seq_idx is not None else q.shape[0])
    if scratch is None:
        scratch = decode_scratch(q.shape[0], nq, nkv, max_ctx, q.device)
    _native.check(_native.lib().sdc_attn_decode(
        q.data_ptr(), out.data_ptr(), cache.data_ptr(), cache.shape[0], block_table.data_ptr(), block_table.shape[1],
        seq_req.data_ptr(), ctx.data_ptr(), None if seq_idx is None else seq_idx.data_ptr(), n, nq, nkv, 128,
        int(max_ctx), float(scale), scratch.data_ptr(), None if row_sq is None else row_sq.data_ptr(),
        None if check is None else check.data_ptr(), _s(q)), "attention decode")
    return out


def reference_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_pos: torch.Tensor) -> torch.Tensor:
    """fp32 reference for one request: q (t, nq, d), k/v (n, nkv, d), causal by absolute positions."""
    nq, nkv = q.shape[1], k.shape[1]
    g = nq // nkv
    kf = k.float().repeat_interleave(g, dim=1)
    vf = v.float().repeat_interleave(g, dim=1)
    s = torch.einsum("thd,nhd->htn", q.float(), kf) / math.sqrt(q.shape[-1])
    keys = torch.arange(k.shape[0], device=q.device)
    mask = keys[None, :] > q_pos[:, None]
    s = s.masked_fill(mask[None], float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.einsum("htn,nhd->thd", p, vf)
