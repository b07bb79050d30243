"""Vocab-parallel cross-entropy.

The LM head is column-parallel over the (padded) vocabulary, so each TP rank
holds logits for a contiguous vocab shard. The loss needs, per token row, the
log-sum-exp over the whole vocabulary and the target's logit. Each rank
reduces its shard to three numbers per row - local max ``m``, local
``sum(exp(l - m))`` and the target logit if the target falls in the shard (0
otherwise) - and ONE all-gather of those ``[3, N]`` stats lets every rank
merge them in rank order:

    M   = max_r m_r
    S   = sum_r s_r * exp(m_r - M)
    lse = M + log S
    loss_row = lse - sum_r t_r

Every rank merges the same gathered numbers in the same order, so the loss is
bitwise identical across the group. The reference issues three all-reduces
(MAX, SUM, SUM) for the same quantities (``dst/loss.py:31-63``); merging the
stats needs one collective and is the same algebra as a flash-attention
softmax merge.

Padded vocab columns (global id >= ``real_vocab``) are masked out: they add
nothing to the denominator and get zero gradient. Backward is local:
``(softmax - onehot) * grad / N`` on this rank's columns. Forward keeps the
shard's ``exp(l - m)`` (it needs it for the sum anyway, and it takes the
place of the fp32 logits), so backward is one per-row rescale by
``exp(m - lse) * grad / N`` - no second exponential pass over ``[N, V]``.

This module is the PyTorch path (CPU, fp32 oracle). On CUDA bf16 the head
GEMM and this reduction are fused into one native kernel
(:mod:`dstraining_b200.ops.fused_head`).
"""

from __future__ import annotations

import torch

from ..parallel.comm import all_gather_dim
from ..parallel.topology import TPContext


def merge_stats(stats: torch.Tensor) -> torch.Tensor:
    """stats: [R, 3, N] rows (m, s, t) from R shards -> (lse [N], target [N])."""
    m, s, t = stats[:, 0], stats[:, 1], stats[:, 2]
    big = m.max(dim=0).values
    total = (s * torch.exp(m - big[None])).sum(dim=0)
    return big + torch.log(total), t.sum(dim=0)


class _VocabParallelCE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, targets, tp, vocab_start, real_vocab):
        in_dtype = logits.dtype
        lf = logits.float()
        n, v_local = lf.shape
        real_cols = min(max(real_vocab - vocab_start, 0), v_local)
        # per-row max over the real columns (-inf for a shard of padding only)
        if real_cols > 0:
            m = lf[:, :real_cols].max(dim=1).values
        else:
            m = torch.full((n,), float("-inf"), dtype=lf.dtype, device=lf.device)
        m_safe = torch.where(torch.isinf(m), torch.zeros_like(m), m)
        e = torch.sub(lf, m_safe[:, None])
        e.exp_()
        if real_cols < v_local:
            e[:, real_cols:] = 0.0
        s = e.sum(dim=1)
        local_t = targets - vocab_start
        in_range = (local_t >= 0) & (local_t < v_local)
        picked = lf.gather(1, local_t.clamp(0, v_local - 1)[:, None]).squeeze(1)
        # a target on a padded column reads as -inf (an infinite loss), as if masked
        picked = torch.where(local_t >= real_cols, torch.full_like(picked, float("-inf")), picked)
        t = torch.where(in_range, picked, torch.zeros_like(picked))
        stats = torch.stack([m_safe, s, t])[None]  # [1, 3, N]
        if tp.enabled:
            stats = all_gather_dim(stats, tp, 0)
        lse, tgt = merge_stats(stats)
        loss = (lse - tgt).mean()
        ctx.save_for_backward(e, m_safe, lse, targets, in_range)
        ctx.vocab_start = vocab_start
        ctx.in_dtype = in_dtype
        return loss

    @staticmethod
    def backward(ctx, grad):
        e, m, lse, targets, in_range = ctx.saved_tensors
        n, v_local = e.shape
        scale = grad / n
        p = e * (torch.exp(m - lse) * scale)[:, None]  # softmax * grad / N
        rows = torch.arange(n, device=e.device)
        cols = (targets - ctx.vocab_start).clamp(0, v_local - 1)
        p[rows, cols] -= in_range.to(p.dtype) * scale
        return p.to(ctx.in_dtype), None, None, None, None


def vocab_parallel_cross_entropy(
    logits: torch.Tensor, targets: torch.Tensor, tp: TPContext, real_vocab: int
) -> torch.Tensor:
    """Mean CE over all tokens. ``logits``: [..., V_local] this rank's shard
    of the padded vocabulary (the whole padded vocabulary when tp=1);
    ``targets``: [...] global ids."""
    v_local = logits.shape[-1]
    return _VocabParallelCE.apply(
        logits.reshape(-1, v_local), targets.reshape(-1), tp, tp.rank * v_local, real_vocab
    )
