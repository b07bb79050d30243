"""The fused tensor-parallel GEMMs run by one process on one GPU.

Every "rank" of an emulated group is a local buffer and every peer flag is
raised before the launch, so no kernel waits for another kernel (the kernels
of several ranks never share a GPU here). What runs is rank 0's launch of
the real kernel - copier threads, tile order, arrival counters, receive slots
and the ordered slot reduction - with local memory in place of NVLink. Used
to check the index arithmetic of every group size up to 8 on a single GPU
(``tests/test_kernels_gpu.py``) and as the small case for ``ncu``
(``utils/kernel_bench.py --op tp_gather / tp_scatter``).
"""

from __future__ import annotations

from typing import List

import torch

from ..ops import native
from ..ops.gemm import EPI_STORE

_RAISED = 1 << 30  # a flag value every bounded wait of a launch accepts


def token_source(tokens: int, seq: int, tp: int):
    """For each global token row: (owning rank, row in the owner's shard), the
    sequence-sharded layout of the fused kernels (rank r holds tokens
    [r T/tp, (r + 1) T/tp) of every batch row)."""
    t = torch.arange(tokens)
    b, pos = t // seq, t % seq
    seq_local = seq // tp
    return pos // seq_local, b * seq_local + pos % seq_local


class GatherEmulation:
    """AG + GEMM as rank 0 of a group of ``tp``: ``y = gather(x_r) W^T`` with
    the shards x_r [tokens / tp, hidden] of every rank as local tensors."""

    def __init__(self, tp: int, tokens: int, hidden: int, ffn: int, seq: int, seed: int = 0):
        g = torch.Generator(device="cuda").manual_seed(seed)
        rows = tokens // tp
        self.tp, self.tokens, self.hidden, self.ffn, self.seq = tp, tokens, hidden, ffn, seq
        self.shards: List[torch.Tensor] = [
            torch.randn(rows, hidden, device="cuda", generator=g).to(torch.bfloat16) for _ in range(tp)
        ]
        self.w = (torch.randn(ffn, hidden, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
        self.flags = torch.full((64,), _RAISED, dtype=torch.int32, device="cuda")
        self.done = torch.zeros(2, dtype=torch.int32, device="cuda")
        self.arrive = torch.zeros(-(-tokens // 128), dtype=torch.int32, device="cuda")
        self.gath = torch.empty(tokens, hidden, dtype=torch.bfloat16, device="cuda")
        self.epoch = 0

    def run(self, precopied: bool = False) -> torch.Tensor:
        """One launch. ``precopied``: every remote block already sits in the
        gather buffer (arrival counters and the copy claim counter set ahead),
        so the copier does nothing - the GEMM part alone, for comparison."""
        self.epoch += 1
        if precopied:
            self.gath.copy_(self.gathered())
            self.arrive.fill_(self.epoch * (self.hidden // 64))
            per_src = (self.tokens // 128) // self.tp
            self.done[1] = (self.tp - 1) * per_src * (self.hidden // 64)
        ptrs = [x.data_ptr() for x in self.shards]
        return native.lib().tp_gemm(
            self.shards[0], False, self.w, False, self.tokens, self.ffn, self.hidden, EPI_STORE, 1, ptrs,
            [self.flags.data_ptr()] * self.tp, self.done, 0, self.seq, self.epoch, gath=self.gath, arrive=self.arrive,
        )[0]

    def gathered(self) -> torch.Tensor:
        """The [tokens, hidden] input every rank's GEMM sees."""
        src, local = token_source(self.tokens, self.seq, self.tp)
        full = torch.empty(self.tokens, self.hidden, dtype=torch.bfloat16, device="cuda")
        for r in range(self.tp):
            sel = (src == r).nonzero().flatten().cuda()
            full[sel] = self.shards[r][local[src == r].cuda()]
        return full


class ScatterEmulation:
    """GEMM + RS as rank 0 of a group of ``tp``: rank 0's partial
    ``h W^T`` [tokens, hidden] goes to every owner's receive slot, then rank
    0's slots are reduced in rank order. The other ranks' slots of rank 0
    hold zeros, so the result is rank 0's own rows of ``h W^T``."""

    def __init__(self, tp: int, tokens: int, hidden: int, ffn: int, seq: int, seed: int = 0):
        g = torch.Generator(device="cuda").manual_seed(seed)
        self.tp, self.tokens, self.hidden, self.ffn, self.seq = tp, tokens, hidden, ffn, seq
        self.rows = tokens // tp
        self.h = torch.randn(tokens, ffn, device="cuda", generator=g).to(torch.bfloat16)
        self.w = (torch.randn(hidden, ffn, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
        self.recv = [torch.zeros(tp * self.rows, hidden, dtype=torch.bfloat16, device="cuda") for _ in range(tp)]
        self.flags = torch.full((64,), _RAISED, dtype=torch.int32, device="cuda")
        self.done = torch.zeros(2, dtype=torch.int32, device="cuda")
        self.epoch = 0

    def run(self) -> torch.Tensor:
        self.epoch += 1
        lib = native.lib()
        ptrs = [x.data_ptr() for x in self.recv]
        fl = [self.flags.data_ptr()] * self.tp
        lib.tp_gemm(self.h, False, self.w, False, self.tokens, self.hidden, self.ffn, EPI_STORE, 3, ptrs, fl,
                    self.done, 0, self.seq, self.epoch)
        return lib.tp_reduce(self.recv[0].view(self.tp, self.rows, self.hidden), self.tp, None, None, fl, self.done,
                             0, self.epoch)

    def own_rows(self) -> torch.Tensor:
        """Row indices (global tokens) that rank 0 owns, in its shard order."""
        src, local = token_source(self.tokens, self.seq, self.tp)
        idx = (src == 0).nonzero().flatten()
        return idx[torch.argsort(local[idx])].cuda()
