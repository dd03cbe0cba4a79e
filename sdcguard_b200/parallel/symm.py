"""Symmetric memory over NVLink for one process per GPU: every rank allocates the same buffers in the same order
(outside torch's caching allocator, so one IPC handle names exactly one buffer), exchanges CUDA IPC handles once
through `torch.distributed` object collectives, and opens its peers' handles on its own device. Peer buffers are
raw device pointers that only this library's kernels dereference (a peer's memory is never handed to cuBLAS, NCCL
or a torch op).

Reference: the reference has no data-path collectives of its own (it observes DTensor/vLLM collectives); this layer
is new.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch
import torch.distributed as dist

from .. import _native

_DT = {torch.bfloat16: ("<V2", 2), torch.float32: ("<f4", 4), torch.int32: ("<i4", 4), torch.int64: ("<i8", 8),
       torch.uint8: ("|u1", 1)}


class _CudaArray:
    """__cuda_array_interface__ view of a raw device pointer (zero copy), for torch.as_tensor."""

    def __init__(self, ptr: int, shape, dtype: torch.dtype):
        typestr = {torch.bfloat16: "<i2", torch.float32: "<f4", torch.int32: "<i4", torch.int64: "<i8",
                   torch.uint8: "|u1"}[dtype]
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


def _wrap(ptr: int, shape, dtype: torch.dtype, device) -> torch.Tensor:
    t = torch.as_tensor(_CudaArray(ptr, shape, dtype), device=device)
    return t.view(torch.bfloat16) if dtype == torch.bfloat16 else t


class SymmetricBuffer:
    def __init__(self, local: torch.Tensor, ptrs: list[int], rank: int, owner=None):
        self.local = local
        self.rank = rank
        self.addr = ptrs                       # every rank's base address, valid on this rank's device
        self._arr = (ctypes.c_ulonglong * len(ptrs))(*ptrs)
        self.ptrs = ctypes.cast(self._arr, ctypes.c_void_p)   # host array for kernel launchers
        self._owner = owner

    @property
    def world(self) -> int:
        return len(self.addr)


class SymmetricHeap:
    """Collective allocator; `alloc` must be called by every rank of `group` with the same arguments."""

    def __init__(self, group: Optional[dist.ProcessGroup] = None, device=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = torch.device(device or torch.cuda.current_device())
        self.buffers: list[SymmetricBuffer] = []
        self._mine: list[int] = []
        self._opened: list[int] = []

    def alloc(self, shape, dtype) -> SymmetricBuffer:
        lib = _native.lib()
        n = 1
        for d in shape:
            n *= int(d)
        nbytes = max(16, n * torch.empty(0, dtype=dtype).element_size())
        with torch.cuda.device(self.device):
            p = ctypes.c_void_p()
            _native.check(lib.sdc_symm_alloc(nbytes, ctypes.byref(p)), "symmetric alloc")
            self._mine.append(p.value)
            hb = ctypes.create_string_buffer(int(lib.sdc_ipc_handle_bytes()))
            _native.check(lib.sdc_ipc_handle(p.value, hb), "ipc handle")
            gathered: list = [None] * self.world
            dist.all_gather_object(gathered, (self.rank, bytes(hb.raw)), group=self.group)
            addrs = [0] * self.world
            for src, h in gathered:
                if src == self.rank:
                    addrs[src] = p.value
                    continue
                q = ctypes.c_void_p()
                _native.check(lib.sdc_ipc_open(h, ctypes.byref(q)), f"ipc open of rank {src}")
                addrs[src] = q.value
                self._opened.append(q.value)
        local = _wrap(p.value, shape, dtype, self.device)
        buf = SymmetricBuffer(local, addrs, self.rank, self)
        self.buffers.append(buf)
        return buf

    def close(self) -> None:
        """Unmap peers and free own buffers (collective: peers must have stopped using them)."""
        lib = _native.lib()
        with torch.cuda.device(self.device):
            torch.cuda.synchronize(self.device)
            for q in self._opened:
                lib.sdc_ipc_close(q)
            for p in self._mine:
                lib.sdc_symm_free(p)
        self._opened, self._mine, self.buffers = [], [], []


class LocalHeap:
    """World size 1 (tests, single GPU): the same interface with no IPC."""

    def __init__(self, device=None):
        self.rank, self.world = 0, 1
        self.device = torch.device(device or torch.cuda.current_device())

    def alloc(self, shape, dtype) -> SymmetricBuffer:
        t = torch.zeros(shape, dtype=dtype, device=self.device)
        return SymmetricBuffer(t, [t.data_ptr()], 0, t)

    def close(self) -> None:
        pass
