"""Fused LM head + (vocab-parallel) cross-entropy on the native path.

Forward runs the head GEMM with a softmax-statistics epilogue: each output
tile reduces its fp32 accumulator rows to (max, sum exp) and picks the target
logit when the target id falls inside the tile, so the loss needs no pass
over the logits. Per-tile stats merge in tile order into per-row stats; under
TP the ``[3, N]`` per-rank stats are all-gathered and merged in rank order
(bitwise identical on every rank): by one peer-memory gather kernel over
NVLink when the group's GPUs can address each other, else one collective.

With sequence parallelism the head's input arrives sequence-sharded: the GEMM
gathers it from the peers itself (gather mode of ``tp_gemm``), the dX of the
backward leaves through the scatter-mode GEMM + slot reduction (the
reduce-scatter), and dW gathers the input again along its K dimension.

Backward turns the saved bf16 logits into ``(softmax - onehot) * grad / N`` in
place and runs the two backward GEMMs (dX = dlogits W, dW = dlogits^T X) on
them. Same math as :mod:`dstraining_b200.ops.cross_entropy`.
"""

from __future__ import annotations

import torch

from ..ops import native
from ..parallel.comm import all_gather_dim, all_reduce_sum, reduce_scatter_dim
from ..parallel.topology import TPContext
from . import tp_fused
from .cross_entropy import merge_stats
from .gemm import EPI_STORE, gemm


class _FusedHeadCE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, targets, tp, real_vocab, seq_parallel):
        lib = native.lib()
        tg = targets.reshape(-1).contiguous()
        v_local = w.shape[0]
        col0 = tp.rank * v_local
        valid = max(0, min(v_local, real_vocab - col0))
        seq = x.shape[1] * tp.world if (seq_parallel and tp.enabled) else x.shape[1]
        fused_sp = seq_parallel and tp.enabled and tp_fused.usable(tp, seq)
        if fused_sp:
            xs = x.reshape(-1, x.shape[-1]).contiguous()  # this rank's sequence shard
            (logits, tmax, tsum, tgt), x2 = tp_fused.ag_gemm(
                id(w), "head.fwd", tp, xs, seq, w, False, tp_fused.EPI_CE_STATS, targets=tg, ce_col0=col0,
                ce_valid=valid,
            )  # x2: the gathered input, kept for dW
        else:
            if seq_parallel and tp.enabled:
                x = all_gather_dim(x, tp, 1)
            x2 = x.reshape(-1, x.shape[-1]).contiguous()
            logits, tmax, tsum, tgt = lib.gemm_ce_stats(x2, w, tg, col0, valid)
        m, s = lib.ce_merge_tiles(tmax, tsum, tg, real_vocab)  # also flags target ids outside the vocabulary
        stats = torch.stack([m, s, tgt])[None]
        if tp.enabled:
            n_rows = stats.shape[-1]
            if tp_fused.usable(tp, seq) and n_rows % 4 == 0:
                # Peer-memory gather of every rank's [3, N] fp32 stats (moved as
                # bytes: [3, 2N] bf16 rows, concatenated in rank order).
                flat = stats.view(3, n_rows).view(torch.bfloat16)
                stats = tp_fused.allgather_rows(id(w), "head.stats", tp, flat, 3 * tp.world)
                stats = stats.view(torch.float32).view(tp.world, 3, n_rows)
            else:
                stats = all_gather_dim(stats, tp, 0)
        lse, tgt_all = merge_stats(stats)
        loss = (lse - tgt_all).mean()
        ctx.save_for_backward(logits, lse, x2, w, tg)
        ctx.meta = (tp, seq_parallel, col0, valid, x.shape, fused_sp, seq, id(w))
        return loss

    @staticmethod
    def backward(ctx, g):
        logits, lse, x2, w, tg = ctx.saved_tensors
        tp, seq_parallel, col0, valid, xshape, fused_sp, seq, k = ctx.meta
        lib = native.lib()
        n = logits.shape[0]
        lib.ce_grad_inplace(logits, lse.contiguous(), tg, col0, valid, g.float().reshape(1).contiguous(), 1.0 / n)
        if fused_sp:
            dx = tp_fused.gemm_rs(k, "head.bwd.rs", tp, logits, seq, w, True).view(xshape)
            dw = gemm(logits, True, x2, True, EPI_STORE)
            return dx, dw, None, None, None, None
        dx = gemm(logits, False, w, True, EPI_STORE).view(xshape)
        dw = gemm(logits, True, x2, True, EPI_STORE)
        if tp.enabled:
            dx = reduce_scatter_dim(dx, tp, 1) if seq_parallel else all_reduce_sum(dx, tp)
        return dx, dw, None, None, None, None


def fused_head_loss(x, w, targets, tp: TPContext, real_vocab: int, seq_parallel: bool):
    return _FusedHeadCE.apply(x, w, targets, tp, real_vocab, seq_parallel)
