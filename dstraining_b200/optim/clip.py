"""Global gradient norm and clipping across tensor- and pipeline-parallel shards.

``grad_norm(model, tp, dp)`` is the L2 norm of the *whole* model's gradient as
a single-process run would see it: TP-sharded parameters (split over ranks by
their layer) contribute their shard, TP-replicated ones (LayerNorm, row
biases, embeddings) are counted once, and every pipeline stage contributes
its own parameters. One all-reduce over all ranks sums the per-rank parts;
data-parallel replicas hold the same (averaged) gradient, so the sum is
divided by the DP degree. Call it after the DP reduction and
``finalize_grads`` (the gradients every optimizer step will use).
``clip_grad_norm`` scales all gradients by ``min(1, max_norm / norm)``.

The fused NVLink DP optimizer consumes gradients inside backward, before a
global norm could exist, so it is not supported there. The reference has no
clipping.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn as nn

from ..parallel.topology import DPContext, TPContext


def _is_sharded(model: nn.Module, name: str) -> bool:
    from ..utils.checkpoint import split_dim

    return split_dim(model, name) is not None


def grad_norm(model: nn.Module, tp: TPContext, dp: DPContext) -> torch.Tensor:
    """Global L2 norm of the gradient (fp32 scalar; a collective over all ranks)."""
    dev = next(model.parameters()).device
    local = torch.zeros((), dtype=torch.float64, device=dev)
    for name, p in model.named_parameters():
        if p.grad is None:
            continue
        sq = p.grad.detach().double().pow(2).sum()
        local += sq if (_is_sharded(model, name) or tp.world == 1) else sq / tp.world
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(local)
        local /= dp.world
    return local.sqrt().float()


def clip_grad_norm(model: nn.Module, max_norm: float, tp: TPContext, dp: DPContext) -> float:
    """Scale every gradient so the global norm is at most ``max_norm``; returns
    the norm before clipping (identical on all ranks)."""
    norm = grad_norm(model, tp, dp)
    coef = torch.clamp(max_norm / (norm + 1e-6), max=1.0)
    for p in model.parameters():
        if p.grad is not None:
            p.grad.mul_(coef.to(p.grad.dtype))
    return float(norm)
