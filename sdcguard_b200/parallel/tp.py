"""Tensor-parallel collectives with carried checksums over NVLink peer memory (`csrc/tp_comm.cu`).

    comm = TPComm(heap, max_rows, hidden)
    # row-parallel GEMM: write the partial output and its seals straight into the symmetric buffers
    gemm.checked_linear(x, w_shard, ..., out=comm.partial(M), seal=comm.partial_seal(M))
    comm.reduce_scatter(M, out=rows_of_this_rank)      # pull peers' partials, verify seals and linearity
    # column-parallel GEMM input: write this rank's rows into the shard buffer, seal them, gather all rows
    comm.shard(R).copy_(...); comm.all_gather(R, out=full)

Sequence parallelism: rows (tokens) are split evenly over ranks; rank d owns rows [d R, (d+1) R).

The NCCL baseline of the same steps is `reduce_scatter_nccl` / `all_gather_nccl` (no checks).
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from .. import _native
from ..numerics import abft

TOL = 4.0     # multiplier on the rounding bound of the linearity check


class TPComm:
    def __init__(self, heap, max_rows: int, hidden: int):
        self.heap = heap
        self.rank, self.world = heap.rank, heap.world
        if max_rows % self.world:
            raise ValueError("max_rows must be a multiple of the world size")
        self.hidden = hidden
        nb = -(-hidden // 128)
        self.nb = nb
        self.max_rows = max_rows
        # rows [0, max_rows): the local partial of the two-step path, or push region 0; [max_rows, 2 max_rows):
        # push region 1 (consecutive fused GEMM + reduce-scatter launches alternate regions)
        self.part = heap.alloc([2 * max_rows, hidden], torch.bfloat16)
        self.part_seal = heap.alloc([2 * max_rows, nb], torch.int32)
        self.shard_buf = heap.alloc([max_rows // self.world, hidden], torch.bfloat16)
        self.shard_seal = heap.alloc([max_rows // self.world, nb], torch.int32)
        self.shard_rss = heap.alloc([max_rows // self.world], torch.float32)   # row_sq of the shard rows
        self.flags = heap.alloc([self.world], torch.int64)
        self.gen = torch.zeros(1, dtype=torch.int64, device=heap.device)
        self.err = torch.zeros(1, dtype=torch.int32, device=heap.device)
        self.state = torch.zeros(2, abft.STATE_COLS, dtype=torch.int64, device=heap.device)   # 0: RS, 1: AG
        self.done = torch.zeros(1, dtype=torch.int32, device=heap.device)     # push-mode GEMM: CTAs finished
        self.norm_done = torch.zeros(1, dtype=torch.int32, device=heap.device)   # shard norm: CTAs finished
        self._inject: Optional[tuple] = None

    def inject_next(self, row: int, col: int, bit: int = 0) -> None:
        """Fault injection: the next reduce_scatter flips one bit of this rank's sealed partial (row, col) before
        the peers read it, as a corrupted transfer would."""
        self._inject = (row, col, bit)

    def _s(self):
        return torch.cuda.current_stream(self.heap.device).cuda_stream

    def partial(self, M: int) -> torch.Tensor:
        return self.part.local[:M]

    def partial_seal(self, M: int) -> torch.Tensor:
        return self.part_seal.local[:M]

    def shard(self, R: int) -> torch.Tensor:
        return self.shard_buf.local[:R]

    def signal(self) -> None:
        _native.check(_native.lib().sdc_tp_signal(self.gen.data_ptr(), self.flags.ptrs, self.world, self.rank,
                                                   self._s()), "tp signal")

    def reduce_scatter(self, M: int, out: torch.Tensor) -> torch.Tensor:
        """Signals that this rank's partial(M) and partial_seal(M) are written, waits for every peer, then sums
        rows [rank R, (rank+1) R) of all partials into out (R, hidden) with seal and linearity checks."""
        R = M // self.world
        if self._inject is not None:
            r, c, bit = self._inject
            self._inject = None
            v = self.part.local.view(torch.int16)[r, c]
            v.bitwise_xor_(1 << bit if bit < 15 else -(1 << 15))
        self.signal()
        _native.check(_native.lib().sdc_tp_reduce_scatter(
            self.part.ptrs, self.part_seal.ptrs, self.gen.data_ptr(), self.flags.local.data_ptr(), self.world,
            self.rank, R, self.hidden, out.data_ptr(), TOL, self.state[0].data_ptr(), self.err.data_ptr(), self._s()),
            "tp reduce-scatter")
        return out

    def can_push(self, M: int) -> bool:
        """The fused GEMM + transfer needs every rank's rows to be whole 128-row tiles."""
        return M % (128 * self.world) == 0 and M <= self.max_rows

    def gemm_reduce_scatter(self, x: torch.Tensor, cw, state: torch.Tensor, slot: int, out: torch.Tensor,
                            row_sq: Optional[torch.Tensor] = None, bn: Optional[int] = None,
                            inject: Optional[tuple] = None) -> torch.Tensor:
        """Row-parallel checked GEMM fused with the reduce-scatter transfer: every output tile of x @ W^T goes from
        the GEMM epilogue straight into the receive buffer of the rank that owns its rows (TMA stores over NVLink,
        with seals), the launch's last CTA raises this rank's flag on every rank, then this rank sums its world
        slots locally with the seal and linearity checks. x: (M, K) with M a multiple of 128 world; out:
        (M / world, N). inject=(row, col, xor) flips an accumulator bit inside the GEMM (caught by its ABFT
        check); `inject_next` flips a bit of this rank's receive buffer after the transfer (caught by the seal)."""
        self.gemm_push(x, cw, state, slot, row_sq=row_sq, bn=bn, inject=inject)
        return self.reduce_local(x.shape[0], out)

    def gemm_push(self, x: torch.Tensor, cw, state: torch.Tensor, slot: int, row_sq: Optional[torch.Tensor] = None,
                  bn: Optional[int] = None, inject: Optional[tuple] = None) -> None:
        import math
        from ..ops import gemm
        M, K = x.shape
        if not self.can_push(M) or K != cw.k or cw.n != self.hidden or x.stride(1) != 1:
            raise ValueError(f"push GEMM needs M % (128 world) == 0 and a ({self.hidden}, {K}) weight")
        lib = _native.lib()
        if row_sq is None:
            row_sq = gemm.row_sqnorm(x)
        dev = x.device
        ws = gemm.workspace(dev, int(lib.sdc_gemm_ws_bytes(M, cw.n)))
        bn = bn or gemm.pick_bn(M, cw.n)
        ir, ic, ix = (-1, -1, 0) if inject is None else (int(inject[0]), int(inject[1]), int(inject[2]))
        s = cw.mask
        _native.check(lib.sdc_gemm_bf16_push(
            x.data_ptr(), x.stride(0), cw.weight.data_ptr(), cw.cs.wc.data_ptr(), M, cw.n, K,
            None if cw.bias is None else cw.bias.data_ptr(), None if cw.cs.bsum is None else cw.cs.bsum.data_ptr(),
            float(cw.cs.bias_max), row_sq.data_ptr(), cw.cs.wstat.data_ptr(), ws.data_ptr(), state.data_ptr(),
            int(slot), s[0], s[1], s[2], s[3], float(abft.Z_ALARM), float(cw.prod_coef), float(cw.out_coef),
            float(abft.ABS_FLOOR), float(math.sqrt(K)), gemm.error_word(dev).data_ptr(), int(bn), ir, ic, ix,
            self.world, self.rank, self.max_rows, self.part.ptrs, self.part_seal.ptrs, self.flags.ptrs, self.gen.data_ptr(),
            self.done.data_ptr(), self._s()), "checked GEMM + reduce-scatter push")

    def reduce_local(self, M: int, out: torch.Tensor) -> torch.Tensor:
        """Waits for every rank's push of the current generation, then sums the world slots of this rank's receive
        buffer (slot r = rows [r R, (r+1) R), written by rank r) into out with the seal and linearity checks."""
        R = M // self.world
        if self._inject is not None:
            r, c, bit = self._inject
            self._inject = None
            torch.cuda.current_stream(self.heap.device).synchronize()    # the push has landed
            off = (int(self.gen.item()) & 1) * self.max_rows
            v = self.part.local.view(torch.int16)[off + r, c]
            v.bitwise_xor_(1 << bit if bit < 15 else -(1 << 15))
        _native.check(_native.lib().sdc_tp_reduce_local(
            self.part.ptrs, self.part_seal.ptrs, self.gen.data_ptr(), self.flags.local.data_ptr(), self.world,
            self.rank, R, self.hidden, self.max_rows, out.data_ptr(), TOL, self.state[0].data_ptr(),
            self.err.data_ptr(), self._s()), "tp reduce (local)")
        return out

    def norm_shard(self, x: torch.Tensor, weight: torch.Tensor, eps: float, residual: Optional[torch.Tensor],
                   resid_out: torch.Tensor, R: int) -> torch.Tensor:
        """add_rmsnorm of this rank's R rows straight into its shard buffer, in one kernel that also writes the
        shard's seals and row_sq and, when every row is written, raises this rank's flag on every rank (the
        all-gather's signal). Follow with all_gather(R, out, sealed=True)."""
        _native.check(_native.lib().sdc_add_rmsnorm_shard(
            x.data_ptr(), None if residual is None else residual.data_ptr(), weight.data_ptr(), float(eps), R,
            self.hidden, self.shard_buf.local.data_ptr(), resid_out.data_ptr(), self.shard_rss.local.data_ptr(),
            self.shard_seal.local.data_ptr(), self.world, self.rank, self.flags.ptrs, self.gen.data_ptr(),
            self.norm_done.data_ptr(), self._s()), "shard norm")
        return self.shard(R)

    def all_gather(self, R: int, out: torch.Tensor, rs_out: Optional[torch.Tensor] = None,
                   sealed: bool = False) -> torch.Tensor:
        """Gathers every rank's shard into out (world R, hidden), checking each row block against its owner's seal.
        Unless `sealed` (the shard came from norm_shard, which sealed it and signalled), seals this rank's shard
        and signals first. rs_out: also gather the shards' row_sq (written by norm_shard)."""
        if not sealed:
            _native.check(_native.lib().sdc_seal_rows(self.shard_buf.local.data_ptr(), self.hidden, R, self.hidden,
                                                      self.shard_seal.local.data_ptr(), self._s()), "seal rows")
            self.signal()
        _native.check(_native.lib().sdc_tp_all_gather(
            self.shard_buf.ptrs, self.shard_seal.ptrs, self.gen.data_ptr(), self.flags.local.data_ptr(), self.world,
            R, self.hidden, out.data_ptr(), self.state[1].data_ptr(), self.err.data_ptr(),
            self.shard_rss.ptrs if rs_out is not None else None, None if rs_out is None else rs_out.data_ptr(),
            self._s()), "tp all-gather")
        return out

    def close(self) -> None:
        """Collective: wait until every rank is done with every buffer, then unmap and free them."""
        torch.cuda.synchronize(self.heap.device)
        if self.world > 1:
            dist.barrier()
        self.heap.close()

    def read_state(self, reset: bool = True) -> dict:
        rows = self.state.cpu().tolist()
        if reset:
            self.state.zero_()
        names = ("reduce_scatter", "all_gather")
        return {n: abft.decode_state_row(r) for n, r in zip(names, rows)} | {"error": int(self.err.item())}


def seal_rows(x: torch.Tensor, seals: torch.Tensor) -> torch.Tensor:
    m, n = x.shape
    _native.check(_native.lib().sdc_seal_rows(x.data_ptr(), x.stride(0), m, n, seals.data_ptr(),
                                              torch.cuda.current_stream(x.device).cuda_stream), "seal rows")
    return seals


# ------------------------------------------------------------------------------------------ NCCL baseline
def _single(group) -> bool:
    """One rank (or no process group at all): every collective is a local copy."""
    return not dist.is_initialized() or dist.get_world_size(group) == 1


def reduce_scatter_nccl(partial: torch.Tensor, out: torch.Tensor, group=None) -> torch.Tensor:
    if _single(group):
        return out.copy_(partial[: out.shape[0]]) if out.data_ptr() != partial.data_ptr() else out
    dist.reduce_scatter_tensor(out, partial, group=group)
    return out


def all_gather_nccl(shard: torch.Tensor, out: torch.Tensor, group=None) -> torch.Tensor:
    if _single(group):
        return out.copy_(shard[: out.shape[0]]) if out.data_ptr() != shard.data_ptr() else out
    dist.all_gather_into_tensor(out, shard, group=group)
    return out
