"""Symmetric heap: one device allocation per rank, mapped into every peer over NVLink (CUDA IPC).

All ranks create the heap with the same size and carve buffers in the same order, so a buffer sits at the same
offset on every rank; ``SymBuf.peers`` is the int64 table of its address on each rank (device tensor, ready to be
passed to kernels) and ``SymBuf.local`` a tensor view of this rank's copy.  Handles are exchanged with one
``all_gather_object`` over the process group.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List

import torch
import torch.distributed as dist

from ..ops._ext import ext

_DT = {torch.bfloat16: "bfloat16", torch.float32: "float32", torch.int32: "int32", torch.int64: "int64",
       torch.uint8: "uint8", torch.float8_e4m3fn: "float8_e4m3fn", torch.float16: "float16"}
_SZ = {torch.bfloat16: 2, torch.float16: 2, torch.float32: 4, torch.int32: 4, torch.int64: 8, torch.uint8: 1,
       torch.float8_e4m3fn: 1}


@dataclass
class SymBuf:
    offset: int
    shape: tuple
    dtype: torch.dtype
    local: torch.Tensor          # this rank's copy
    peers: torch.Tensor          # int64 [world] device addresses of every rank's copy
    peer_addrs: List[int]

    def peer_view(self, r: int, device) -> torch.Tensor:
        return ext().tensor_from_ptr(self.peer_addrs[r], list(self.shape), _DT[self.dtype], device.index or 0)


class SymmHeap:
    def __init__(self, nbytes: int, rank: int, world: int, group=None, device=None):
        self.rank, self.world, self.group = rank, world, group
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.nbytes = int(nbytes)
        e = ext()
        self.base = e.symm_malloc(self.nbytes)
        handle = e.symm_ipc_handle(self.base)
        handles = [None] * world
        dist.all_gather_object(handles, handle, group=group)
        self.peer_base = [self.base if r == rank else e.symm_ipc_open(handles[r]) for r in range(world)]
        self.off = 0
        self._closed = False

    def alloc(self, shape, dtype) -> SymBuf:
        n = 1
        for s in shape:
            n *= int(s)
        size = n * _SZ[dtype]
        off = (self.off + 255) // 256 * 256
        if off + size > self.nbytes:
            raise RuntimeError(f"symmetric heap exhausted ({off + size} > {self.nbytes} bytes)")
        self.off = off + size
        addrs = [b + off for b in self.peer_base]
        local = ext().tensor_from_ptr(addrs[self.rank], [int(s) for s in shape], _DT[dtype], self.device.index or 0)
        peers = torch.tensor(addrs, dtype=torch.int64, device=self.device)
        return SymBuf(off, tuple(int(s) for s in shape), dtype, local, peers, addrs)

    def close(self):
        if self._closed:
            return
        e = ext()
        for r, p in enumerate(self.peer_base):
            if r != self.rank:
                e.symm_ipc_close(p)
        e.symm_free(self.base)
        self._closed = True
