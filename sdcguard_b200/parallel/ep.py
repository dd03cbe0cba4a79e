"""Expert-parallel all-to-all with carried checksums over NVLink peer memory (`csrc/ep_comm.cu`), and the router.

    comm = EPComm(heap, max_tokens, hidden, experts, top_k)
    ids, wts = router_topk(logits, top_k)                  # softmax, top-k, renormalise (Mixtral)
    x_g, row_sq, gband, gcount = comm.dispatch_grouped(x, ids)   # this rank's expert rows on 128-row bands
    y_g = grouped checked GEMMs (gband, gcount)           # models.moe: both expert GEMMs, one launch each
    y = comm.combine(y_g, wts)                             # rows back to their tokens, weighted sum over k

`dispatch` (compact rows and host-side offsets, one device-to-host read) is kept for tools that want the counts.

Every row carries its seals (exact 32-bit hash per 128 columns) through both transfers; the receiving side
re-hashes the bits that arrived. Results fold into `state` rows 0 (dispatch) and 1 (combine).

The NCCL baseline of the same exchange is `all_to_all_nccl` (torch.distributed.all_to_all_single, no checks).
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from .. import _native
from ..numerics import abft


def _s(dev):
    return torch.cuda.current_stream(dev).cuda_stream


def router_topk(logits: torch.Tensor, k: int, ids: Optional[torch.Tensor] = None, wts: Optional[torch.Tensor] = None,
                rows: Optional[torch.Tensor] = None, check: Optional[torch.Tensor] = None):
    """logits (T, E) bf16 -> ids (T, k) int32, weights (T, k) fp32. With rows and check: exact replay of the
    sampled tokens against the stored ids / weights."""
    T, E = logits.shape
    dev = logits.device
    if ids is None:
        ids = torch.empty(T, k, dtype=torch.int32, device=dev)
    if wts is None:
        wts = torch.empty(T, k, dtype=torch.float32, device=dev)
    _native.check(_native.lib().sdc_router_topk(
        logits.data_ptr(), logits.stride(0), T, E, k, ids.data_ptr(), wts.data_ptr(),
        None if rows is None else rows.data_ptr(), 0 if rows is None else rows.numel(),
        None if check is None else check.data_ptr(), _s(dev)), "router top-k")
    return ids, wts


class EPComm:
    def __init__(self, heap, max_tokens: int, hidden: int, experts: int, top_k: int):
        self.heap = heap
        self.rank, self.world = heap.rank, heap.world
        if experts % self.world:
            raise ValueError("experts must divide evenly over the ranks")
        self.epr = experts // self.world
        self.experts, self.k, self.H = experts, top_k, hidden
        self.cap = max_tokens                  # a token sends at most one row to each expert
        self.nb = -(-hidden // 128)
        rows = self.world * self.epr * self.cap
        dev = heap.device
        self.d_rows = heap.alloc([rows, hidden], torch.bfloat16)
        self.d_seal = heap.alloc([rows, self.nb], torch.int32)
        self.d_meta = heap.alloc([rows], torch.int32)
        self.d_cnt = heap.alloc([self.world * self.epr], torch.int32)
        self.c_rows = heap.alloc([rows, hidden], torch.bfloat16)
        self.c_seal = heap.alloc([rows, self.nb], torch.int32)
        self.flags = heap.alloc([self.world], torch.int64)
        self.gen = torch.zeros(1, dtype=torch.int64, device=dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        self.counts = torch.zeros(self.world * self.epr, dtype=torch.int32, device=dev)
        self.plan = torch.empty(max_tokens * top_k, 2, dtype=torch.int32, device=dev)
        grows = rows + self.epr * 128          # the grouped layout pads each expert to whole 128-row bands
        self.recv = torch.zeros(grows, hidden, dtype=torch.bfloat16, device=dev)   # rows past the bands in use stay finite
        self.map = torch.empty(grows, dtype=torch.int32, device=dev)
        self.row_sq = torch.zeros(grows, dtype=torch.float32, device=dev)
        self.gband = torch.zeros(grows // 128 + 1, dtype=torch.int32, device=dev)
        self.gcount = torch.zeros(1, dtype=torch.int32, device=dev)
        self.offs = torch.zeros(self.epr + 1, dtype=torch.int32, device=dev)
        self.state = torch.zeros(2, abft.STATE_COLS, dtype=torch.int64, device=dev)   # 0 dispatch, 1 combine
        self._inj_d = (-1, 0, 0)
        self._inj_c = (-1, 0, 0)
        self.T = 0

    def inject_dispatch(self, pair: int, col: int, bit: int) -> None:
        """Flip `bit` (0-15) of element `col` of the row sent for (token, k) pair index `pair` after sealing."""
        self._inj_d = (pair, col, bit)

    def inject_combine(self, row: int, col: int, bit: int) -> None:
        """Flip a bit of compact expert-output row `row` as it is pushed back."""
        self._inj_c = (row, col, bit)

    def _send(self, x: torch.Tensor, ids: torch.Tensor) -> None:
        T = x.shape[0]
        if T > self.cap:
            raise ValueError(f"{T} tokens exceed the capacity {self.cap}")
        self.T = T
        dev = x.device
        lib = _native.lib()
        self.counts.zero_()
        inj = self._inj_d
        self._inj_d = (-1, 0, 0)
        _native.check(lib.sdc_ep_dispatch(
            x.data_ptr(), ids.data_ptr(), T, self.k, self.H, self.world, self.rank, self.epr, self.cap,
            self.counts.data_ptr(), self.plan.data_ptr(), self.d_rows.ptrs, self.d_seal.ptrs, self.d_meta.ptrs,
            self.d_cnt.ptrs, self.flags.ptrs, self.gen.data_ptr(), inj[0], inj[1], inj[2], _s(dev)), "ep dispatch")

    def dispatch_grouped(self, x: torch.Tensor, ids: torch.Tensor):
        """x (T, H) bf16, ids (T, k) int32 -> (rows, row_sq, gband, gcount): this rank's expert rows grouped by
        local expert, each expert's rows starting on a 128-row band and padded with zero rows, their sums of
        squares, the band -> local expert table and the number of bands in use (device tensors; nothing is read
        back). The input of `ops.gemm.checked_linear_grouped`."""
        self._send(x, ids)
        dev = x.device
        _native.check(_native.lib().sdc_ep_receive_grouped(
            self.d_rows.local.data_ptr(), self.d_seal.local.data_ptr(), self.d_cnt.local.data_ptr(),
            self.gen.data_ptr(), self.flags.local.data_ptr(), self.world, self.rank, self.epr, self.cap, self.H,
            self.recv.data_ptr(), self.map.data_ptr(), self.offs.data_ptr(), self.gband.data_ptr(),
            self.gcount.data_ptr(), self.row_sq.data_ptr(), self.state[0].data_ptr(), self.err.data_ptr(), _s(dev)),
            "ep receive (grouped)")
        return self.recv, self.row_sq, self.gband, self.gcount

    def dispatch(self, x: torch.Tensor, ids: torch.Tensor) -> tuple[torch.Tensor, list[int]]:
        """x (T, H) bf16, ids (T, k) int32 -> rows for this rank's experts (compact, grouped by local expert) and
        the per-expert row offsets (host list; one device->host read)."""
        self._send(x, ids)
        dev = x.device
        lib = _native.lib()
        _native.check(lib.sdc_ep_receive(
            self.d_rows.local.data_ptr(), self.d_seal.local.data_ptr(), self.d_cnt.local.data_ptr(),
            self.gen.data_ptr(), self.flags.local.data_ptr(), self.world, self.rank, self.epr, self.cap, self.H,
            self.recv.data_ptr(), self.map.data_ptr(), self.offs.data_ptr(), self.state[0].data_ptr(),
            self.err.data_ptr(), _s(dev)), "ep receive")
        offs = self.offs.tolist()
        return self.recv[: offs[-1]], offs

    def combine(self, y: torch.Tensor, wts: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """y: expert outputs in the compact order of `dispatch`; wts (T, k) fp32 -> (T, H) bf16."""
        dev = y.device
        lib = _native.lib()
        T = self.T
        if out is None:
            out = torch.empty(T, self.H, dtype=torch.bfloat16, device=dev)
        inj = self._inj_c
        self._inj_c = (-1, 0, 0)
        _native.check(lib.sdc_ep_combine_push(
            y.data_ptr(), self.map.data_ptr(), self.offs.data_ptr(), y.shape[0], self.world, self.rank, self.epr,
            self.cap, self.H, self.c_rows.ptrs, self.c_seal.ptrs, self.flags.ptrs, self.gen.data_ptr(), inj[0],
            inj[1], inj[2], _s(dev)), "ep combine push")
        _native.check(lib.sdc_ep_combine(
            self.c_rows.local.data_ptr(), self.c_seal.local.data_ptr(), self.plan.data_ptr(), wts.data_ptr(),
            self.gen.data_ptr(), self.flags.local.data_ptr(), T, self.k, self.H, self.world, self.rank, self.epr,
            self.cap, out.data_ptr(), self.state[1].data_ptr(), self.err.data_ptr(), _s(dev)), "ep combine")
        return out

    def read_state(self, reset: bool = True) -> dict:
        rows = self.state.cpu().tolist()
        if reset:
            self.state.zero_()
        out = {}
        for name, r in zip(("dispatch", "combine"), rows):
            d = abft.decode_state_row(r)
            if d["z"] > 0:
                d["row"], d["block"] = divmod(d["flat"], self.nb)
                d["src_or_expert_rank"], rem = divmod(d["row"], self.epr * self.cap)
                d["expert"], d["slot"] = divmod(rem, self.cap)
            out[name] = d
        out["error"] = int(self.err.item())
        return out

    def close(self) -> None:
        torch.cuda.synchronize(self.heap.device)
        if self.world > 1:
            dist.barrier()
        self.heap.close()


def all_to_all_nccl(x: torch.Tensor, ids: torch.Tensor, experts: int, group=None):
    """Baseline: the same exchange with torch.distributed.all_to_all_single (no checks). Returns the received rows
    (grouped by source rank), the send order and the split sizes."""
    world = dist.get_world_size(group)
    epr = experts // world
    dest = (ids.long() // epr).view(-1)
    order = torch.argsort(dest, stable=True)
    send = x.repeat_interleave(ids.shape[1], dim=0)[order]
    sc = torch.bincount(dest, minlength=world)
    rc = torch.empty_like(sc)
    dist.all_to_all_single(rc, sc, group=group)
    scl, rcl = sc.tolist(), rc.tolist()
    recv = torch.empty(sum(rcl), x.shape[1], dtype=x.dtype, device=x.device)
    dist.all_to_all_single(recv, send, rcl, scl, group=group)
    return recv, order, scl, rcl
