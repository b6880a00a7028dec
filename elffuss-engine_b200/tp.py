"""Host side of the tensor-parallel decode collectives (ef_tp_* in the C
library): exchange buffers of this rank, their CUDA IPC handles swapped over
the torch.distributed process group, and the one-shot all-reduce / all-gather
calls the decoders use between their kernels (captured in their CUDA graphs).

One process per GPU of one node; every rank makes the same calls in the same
order. Data larger than `max_bytes` per rank (a long prompt's activations)
goes through torch.distributed (NCCL) instead.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from ._lib import EfError, check, lib

HANDLE_BYTES = 64


class TPComm:
    def __init__(self, ops, rank: int, world: int, max_bytes: int = 1 << 20, timeout_s: float = 2.0, group=None):
        self.ops, self.rank, self.world, self.max_bytes = ops, rank, world, max_bytes
        L, h = lib(), ops.ctx.bind()
        self.tp = ctypes.c_void_p()
        check(L.ef_tp_create(h, rank, world, max_bytes, ctypes.c_double(timeout_s), ctypes.byref(self.tp)), h)
        mine = ctypes.create_string_buffer(HANDLE_BYTES)
        check(L.ef_tp_handle(h, self.tp, mine), h)
        allh = [None] * world
        dist.all_gather_object(allh, bytes(mine.raw), group=group)
        blob = ctypes.create_string_buffer(b"".join(allh), HANDLE_BYTES * world)
        check(L.ef_tp_connect(h, self.tp, blob), h)
        dist.barrier(group=group)          # every rank mapped before the first call

    def fits(self, t: torch.Tensor) -> bool:
        return t.numel() * t.element_size() <= self.max_bytes

    def all_reduce(self, t: torch.Tensor):
        """In-place sum over the ranks (f32, contiguous), in rank order."""
        if not self.fits(t):
            dist.all_reduce(t)
            return
        h = self.ops.ctx.bind()
        check(lib().ef_allreduce_sum(h, self.tp, ctypes.c_void_p(t.data_ptr()), t.numel()), h)

    def all_gather(self, dst: torch.Tensor, src: torch.Tensor):
        """dst = the ranks' src concatenated in rank order (4-byte elements)."""
        h = self.ops.ctx.bind()
        check(lib().ef_allgather(h, self.tp, ctypes.c_void_p(src.data_ptr()), src.numel() * src.element_size(),
                                 ctypes.c_void_p(dst.data_ptr())), h)

    def status(self) -> int:
        h = self.ops.ctx.bind()
        return lib().ef_tp_status(h, self.tp)

    def close(self):
        if getattr(self, "tp", None) is not None and self.tp.value:
            lib().ef_tp_destroy(self.ops.ctx.h, self.tp)
            self.tp = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
