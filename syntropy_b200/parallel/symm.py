"""Symmetric-memory region: the same byte layout allocated on every rank and mapped into
every other rank's address space with CUDA IPC, so kernels address peers' buffers with
plain loads and stores over NVLink (csrc/cpu/symm.cpp)."""
from __future__ import annotations

import torch
import torch.distributed as dist

from .._ext import ext
from .dist import DistContext


class SymmetricRegion:
    def __init__(self, ctx: DistContext, nbytes: int):
        self.ctx = ctx
        self.nbytes = nbytes
        self.local, handle = ext().symm_alloc(nbytes)
        handles = [None] * ctx.world
        dist.all_gather_object(handles, handle.numpy().tobytes(), group=ctx.cpu_group)
        self.ptrs = []
        self._opened = []
        for r, hb in enumerate(handles):
            if r == ctx.rank:
                self.ptrs.append(self.local.data_ptr())
            else:
                p = ext().symm_open(torch.frombuffer(bytearray(hb), dtype=torch.uint8))
                self._opened.append(p)
                self.ptrs.append(p)
        self.peers = torch.tensor(self.ptrs, dtype=torch.int64, device=ctx.device)
        dist.barrier(group=ctx.cpu_group)

    def view(self, offset: int, numel: int, dtype) -> torch.Tensor:
        """Local tensor view at a byte offset."""
        es = torch.tensor([], dtype=dtype).element_size()
        return self.local[offset: offset + numel * es].view(dtype)

    def close(self):
        for p in self._opened:
            try:
                ext().symm_close(p)
            except Exception:
                pass
        self._opened = []
