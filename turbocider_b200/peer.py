"""Buffers shared by the ranks of one box and the fused all-gather barrier.

N-column sharding (each rank holds a column range of every quantised weight)
needs every rank's output columns on every rank.  Here the GEMM writes them
there itself: `PeerGroup.alloc` makes a buffer on every rank and maps all of
them into every process (CUDA IPC handles exchanged through
torch.distributed); `turbocider_b200.cuda.qlinear(..., peers=...)` stores each
output into this rank's buffer and into the same columns of the others
(NVLink peer stores from the epilogue); `PeerGroup.barrier(stream)` then makes
every rank's stream wait until all ranks have finished (a bounded device-side
flag barrier, tc_cuda_peer_barrier).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import cuda as tcc


class _CudaArray:
    """Minimal __cuda_array_interface__ holder so torch can view a raw pointer."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


class SymmetricBuffer:
    """One device buffer per rank; `ptrs[r]` is rank r's buffer as mapped in
    this process (`ptrs[rank]` is the local one)."""

    def __init__(self, group: "PeerGroup", nbytes: int):
        import torch.distributed as dist
        self.group, self.nbytes = group, nbytes
        lib = tcc.lib()
        local = C.c_void_p()
        handle = (C.c_uint8 * 64)()
        tcc._check(lib.tc_cuda_peer_alloc(group.ctx.handle, nbytes, C.byref(local), handle))
        self.local = local.value
        handles = [None] * group.world
        dist.all_gather_object(handles, bytes(handle), group=group.pg)
        self.ptrs, self._opened = [], []
        for r, h in enumerate(handles):
            if r == group.rank:
                self.ptrs.append(self.local)
                continue
            p = C.c_void_p()
            hb = (C.c_uint8 * 64).from_buffer_copy(h)
            tcc._check(lib.tc_cuda_peer_open(group.ctx.handle, hb, C.byref(p)))
            self.ptrs.append(p.value)
            self._opened.append(p.value)

    def tensor(self, shape, dtype):
        """torch view of the local buffer."""
        import torch
        code = {torch.float32: "<f4", torch.float16: "<f2", torch.bfloat16: "<u2", torch.uint32: "<u4",
                torch.uint8: "|u1"}[dtype]
        count = int(np.prod(shape))
        assert count * torch.tensor([], dtype=dtype).element_size() <= self.nbytes
        t = torch.as_tensor(_CudaArray(self.local, shape, code), device=f"cuda:{self.group.ctx.device}")
        return t.view(torch.bfloat16) if dtype == torch.bfloat16 else t

    def unmap(self):
        """Close this process's mappings of the other ranks' buffers."""
        lib = tcc.lib()
        for p in self._opened:
            lib.tc_cuda_peer_close(self.group.ctx.handle, C.c_void_p(p))
        self._opened = []

    def free(self):
        if self.local:
            tcc.lib().tc_cuda_peer_free(self.group.ctx.handle, C.c_void_p(self.local))
            self.local = 0


class PeerGroup:
    """The ranks of a torch.distributed process group (one per GPU, all on one
    box) as seen by the fused all-gather."""

    def __init__(self, ctx: tcc.Context, pg=None, timeout_us: int = 1_000_000):
        import torch.distributed as dist
        self.ctx, self.pg = ctx, pg
        self.world = dist.get_world_size(pg)
        self.rank = dist.get_rank(pg)
        if self.world > 8:
            raise ValueError("the fused all-gather spans at most 8 ranks")
        self.timeout_us = timeout_us
        self.flags = SymmetricBuffer(self, 4 * self.world)
        self.epoch = 0
        self.buffers = [self.flags]

    def alloc(self, nbytes: int) -> SymmetricBuffer:
        buf = SymmetricBuffer(self, nbytes)
        self.buffers.append(buf)
        return buf

    def peers_of(self, buf: SymmetricBuffer, byte_offset: int = 0) -> list:
        """The other ranks' copies of `buf` (+ byte_offset), for qlinear(peers=...)."""
        return [p + byte_offset for r, p in enumerate(buf.ptrs) if r != self.rank]

    def push(self, buf: SymmetricBuffer, byte_offset: int, nbytes: int, stream=None):
        """All-gather step: copy bytes [byte_offset, +nbytes) of this rank's
        `buf` into the same bytes of every other rank's `buf`
        (tc_cuda_peer_push, enqueued on `stream`; by the copy engines, or by
        the SMs' push kernel after Context.set_push_kernel).  Rank r sends to r+1, r+2, ...
        in turn, so at any moment every rank receives from a different sender.
        Completion on every rank: `barrier` on the same stream."""
        order = [(self.rank + i) % self.world for i in range(1, self.world)]
        dst = (C.c_void_p * max(1, len(order)))(*[buf.ptrs[r] + byte_offset for r in order])
        tcc._check(tcc.lib().tc_cuda_peer_push(self.ctx.handle, C.c_void_p(buf.local + byte_offset), dst, len(order),
                                               nbytes, 1, nbytes, nbytes, tcc._stream_ptr(stream)))

    def barrier(self, stream=None):
        """Every rank's `stream` waits until all ranks reached this barrier."""
        self.epoch += 1
        fl = (C.c_void_p * self.world)(*self.flags.ptrs)
        tcc._check(tcc.lib().tc_cuda_peer_barrier(self.ctx.handle, fl, self.world, self.rank, self.epoch,
                                                  self.timeout_us, tcc._stream_ptr(stream)))

    def close(self):
        """Unmap the peers' buffers everywhere, then free the local ones (no rank
        frees a buffer another rank still maps)."""
        import torch
        import torch.distributed as dist
        torch.cuda.synchronize(self.ctx.device)
        for b in self.buffers:
            b.unmap()
        dist.barrier(self.pg)
        for b in self.buffers:
            b.free()
        self.buffers = []
