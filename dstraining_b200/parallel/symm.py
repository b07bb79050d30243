"""Peer memory over NVLink: equal-sized buffers on every rank of a group,
mapped into every other rank's address space.

``PeerBuffer(nbytes, ctx, device)`` allocates a zeroed, IPC-exportable device
buffer on each rank, exchanges the CUDA IPC handles over the group and maps
each peer's buffer (``cudaIpcOpenMemHandle``). ``ptrs[r]`` is rank r's buffer as
seen from this process; ``local`` is this rank's own buffer as a uint8
tensor. Kernels receive the pointer table and load/store peers' memory
directly (no NCCL, no cluster-shared TMA copies). Collective: every rank of the group must
construct the same buffers in the same order.
"""

from __future__ import annotations

from typing import List

import torch
import torch.distributed as dist

from ..ops import native
from .topology import TPContext


class PeerBuffer:
    """Equal-sized device buffers on every rank of ``ctx``, each mapped into every
    other rank (CUDA IPC); ``ptrs[r]`` is rank r's buffer as seen from here.
    Collective: all ranks construct the same buffers in the same order."""

    def __init__(self, nbytes: int, ctx: TPContext, device: torch.device):
        lib = native.lib()
        self.ctx = ctx
        self.device = device
        self._opened: List[int] = []
        self.nbytes = nbytes
        self.local, handle = lib.symm_alloc(int(nbytes), device.index)
        handles: List = [None] * ctx.world
        if ctx.enabled:
            dist.all_gather_object(handles, bytes(handle.tolist()), group=ctx.group)
        else:
            handles[0] = bytes(handle.tolist())
        self.ptrs: List[int] = []
        self._opened: List[int] = []
        for r in range(ctx.world):
            if r == ctx.rank:
                self.ptrs.append(self.local.data_ptr())
            else:
                h = torch.tensor(list(handles[r]), dtype=torch.uint8)
                p = lib.symm_open(h, device.index)
                self.ptrs.append(p)
                self._opened.append(p)

    def view(self, dtype: torch.dtype) -> torch.Tensor:
        return self.local.view(dtype)

    def close(self) -> None:
        lib = native.lib()
        for p in self._opened:
            lib.symm_close(p, self.device.index)
        self._opened = []
