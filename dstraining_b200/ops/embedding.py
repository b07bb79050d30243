"""Token + position embedding.

``x[b, t] = wte[idx[b, t]] + wpe[t]``. With sequence parallelism the result
enters the first sequence-sharded region, so on the native path the kernel
emits only this rank's sequence chunk (rows ``[rank*T/tp, (rank+1)*T/tp)``)
instead of building the full ``[B, T, C]`` tensor and slicing it.

Backward: the sequence-sharded gradient is all-gathered along the sequence
(the ``scatter`` operator's backward), then a deterministic scatter-add
builds the wte/wpe gradients: the token ids are stably sorted, and one warp
per distinct id sums that id's gradient rows in token order into an fp32
register accumulator (no atomics, so the summation order is fixed).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from . import native
from ..parallel.comm import all_gather_dim, scatter_along_seq
from ..parallel.topology import TPContext


class _EmbedFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, idx, wte, wpe, tp, seq_parallel):
        b, t = idx.shape
        t0, tl = 0, t
        if seq_parallel and tp.enabled:
            tl = t // tp.world
            t0 = tp.rank * tl
        out = native.lib().embedding_fwd(idx, wte, wpe, t0, tl)
        ctx.save_for_backward(idx)
        ctx.meta = (tp, seq_parallel, wte.shape[0], wpe.shape[0])
        return out

    @staticmethod
    def backward(ctx, dy):
        (idx,) = ctx.saved_tensors
        tp, seq_parallel, vocab, block = ctx.meta
        if seq_parallel and tp.enabled:
            dy = all_gather_dim(dy, tp, 1)
        dwte, dwpe = native.lib().embedding_bwd(dy.contiguous(), idx, vocab, block)
        return None, dwte, dwpe, None, None


def embed_tokens(idx, wte, wpe, tp: TPContext, seq_parallel: bool):
    b, t = idx.shape
    if seq_parallel and tp.enabled and t % tp.world:
        raise ValueError(f"seq len {t} not divisible by tp {tp.world}")
    if native.active(wte, wpe) and idx.is_cuda:
        return _EmbedFn.apply(idx, wte, wpe, tp, seq_parallel)
    pos = torch.arange(t, device=idx.device)
    x = F.embedding(idx, wte) + F.embedding(pos, wpe)
    if seq_parallel:
        x = scatter_along_seq(x, tp)
    return x
