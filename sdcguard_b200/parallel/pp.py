"""Pipeline parallelism with sealed stage-to-stage transfers on NCCL point-to-point, overlapped with compute.

Each stage runs a contiguous range of decoder layers (`CheckedDecoder.forward(layer_range=..., hidden=..., last=...)`)
over a sequence of microbatches. Between stages the residual-stream state (x, resid) moves with `isend` / `irecv`
(NCCL over NVLink on GPUs, gloo on CPU), together with its seals: the exact 32-bit hash of every (row, 128-column
block) that the sender computes from the bits it sends (`seal_rows` kernel) and the receiver recomputes from the bits
it got (`sdc_seal_verify`, a mismatch goes to the stage's state row with its row, block and sending stage). Sends are
asynchronous: stage s starts microbatch m + 1 while m is on the wire, and stage s + 1 computes m while s computes
m + 1. Verification is enqueued on the compute stream after the receive, with no host synchronisation.

    comm = SealedP2P(rank, world, device)          # one process per stage
    outs = run_stage(model, comm, metas, cache)     # logits on the last stage, [] elsewhere

Reference: the reference has no pipeline parallelism (`stack.py:23-26` records vLLM's pipeline size only); the plan
is NCCL p2p send/recv, overlapped, with the checks carried (a new component).
"""
from __future__ import annotations

from typing import Optional, Sequence

import torch
import torch.distributed as dist

from .. import _native
from ..numerics import abft


def stage_layers(n_layers: int, stage: int, stages: int) -> tuple[int, int]:
    """Contiguous split of n_layers over stages, the first stages taking one more when it does not divide."""
    q, r = divmod(n_layers, stages)
    lo = stage * q + min(stage, r)
    return lo, lo + q + (1 if stage < r else 0)


class SealedP2P:
    """Sealed point-to-point transfers between pipeline stages."""

    def __init__(self, rank: int, world: int, device, group=None):
        self.rank, self.world, self.group = rank, world, group
        self.device = torch.device(device)
        self.state = torch.zeros(abft.STATE_COLS, dtype=torch.int64, device=self.device)
        self._inject: Optional[tuple] = None

    def inject_next(self, row: int, col: int, bit: int = 3) -> None:
        """Fault injection: the next send flips one bit of its first tensor after sealing (corruption in transit)."""
        self._inject = (row, col, bit)

    def _seal(self, x: torch.Tensor) -> torch.Tensor:
        m, n = x.shape
        s = torch.empty(m, -(-n // 128), dtype=torch.int32, device=x.device)
        if x.is_cuda:
            from .tp import seal_rows
            return seal_rows(x, s)
        from ..ops.gemm import seal_reference
        return seal_reference(x)

    def send(self, tensors: Sequence[torch.Tensor], dst: int) -> list:
        works = []
        for k, t in enumerate(tensors):
            seals = self._seal(t)
            if k == 0 and self._inject is not None:
                r, c, bit = self._inject
                self._inject = None
                t = t.clone()
                v = t.view(torch.int16)[r, c]
                v.bitwise_xor_(1 << bit if bit < 15 else -(1 << 15))
            works.append(dist.isend(t.contiguous(), dst, group=self.group))
            works.append(dist.isend(seals, dst, group=self.group))
            works.append(t)          # kept alive until the sends complete
            works.append(seals)
        return works

    def recv(self, shapes: Sequence[tuple], src: int) -> list[torch.Tensor]:
        outs, works = [], []
        for shp in shapes:
            t = torch.empty(shp, dtype=torch.bfloat16, device=self.device)
            s = torch.empty(shp[0], -(-shp[1] // 128), dtype=torch.int32, device=self.device)
            works += [dist.irecv(t, src, group=self.group), dist.irecv(s, src, group=self.group)]
            outs.append((t, s))
        for w in works:
            w.wait()
        res = []
        for t, s in outs:
            self.verify(t, s, src)
            res.append(t)
        return res

    def verify(self, x: torch.Tensor, want: torch.Tensor, src: int) -> None:
        m, n = x.shape
        self.nb = -(-n // 128)
        if x.is_cuda:
            _native.check(_native.lib().sdc_seal_verify(
                x.data_ptr(), x.stride(0), m, n, want.data_ptr(), int(src), self.state.data_ptr(),
                torch.cuda.current_stream(x.device).cuda_stream), "seal verify")
            return
        from ..ops.gemm import seal_reference
        got = seal_reference(x)
        self.state[2] += 1
        bad = (got != want).nonzero()
        if bad.numel():
            r, b = int(bad[0, 0]), int(bad[0, 1])
            nb = want.shape[1]
            flat = (r * nb + b) * 8 + int(src)
            key = (0x7f800000 << 32) | (flat & 0xFFFFFFFF)
            self.state[0] = max(int(self.state[0]), key)

    def read_state(self, reset: bool = True) -> dict:
        row = self.state.cpu().tolist()
        if reset:
            self.state.zero_()
        d = abft.decode_state_row(row)
        if d["z"] > 0:
            rb, d["peer"] = divmod(d["flat"], 8)
            d["row"], d["block"] = divmod(rb, getattr(self, "nb", 1))
        return d


def run_stage(model, comm: SealedP2P, metas: Sequence, cache: torch.Tensor, stages: Optional[int] = None) -> list:
    """Pipelined forward of every microbatch through this stage's layers; returns the last stage's logits (a list per
    microbatch), [] on other stages. metas: the microbatches' StepMeta (same on every stage); cache: this stage's
    KV layers."""
    stages = stages or comm.world
    stage = comm.rank
    lo, hi = stage_layers(len(model.layers), stage, stages)
    H = model.cfg.hidden
    outs, pending = [], []
    for meta in metas:
        T = meta.tokens.shape[0]
        hidden = None
        if stage > 0:
            x, r = comm.recv([(T, H), (T, H)], stage - 1)
            hidden = (x, r)
        if stage < stages - 1:
            x, r = model.forward(meta, cache, layer_range=(lo, hi), hidden=hidden, last=False)
            pending += comm.send([x.clone(), r.clone()], stage + 1)   # the activation buffers are reused next
        else:
            outs.append(model.forward(meta, cache, layer_range=(lo, hi), hidden=hidden).clone())
    for w in pending:
        if hasattr(w, "wait"):
            w.wait()
    return outs
