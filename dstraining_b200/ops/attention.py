"""Causal self-attention core.

Input is the fused QKV projection output ``[B, T, h * 3 * d]`` laid out
head-major (``[head0: q|k|v, head1: q|k|v, ...]``, the reference's layout,
``dst/model.py:133-161``), so a column split of the projection hands each TP
rank whole heads. Output is ``[B, T, h * d]``.

* CUDA bf16: the hand-written sm_100a flash-attention kernels read Q, K and V
  straight out of the QKV buffer (strided, no split/transposes), keep the
  running softmax on chip and save only the per-row log-sum-exp for
  backward; backward is deterministic (no atomics), so recomputed and stored
  runs give bit-identical gradients.
* otherwise: :func:`core_attention`, the materialised reference algorithm,
  optionally wrapped in :func:`recompute`.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from . import native
from .recompute import recompute


def core_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """softmax(q k^T / sqrt(d) + causal mask) v with the s x s score matrix
    materialised (the memory that selective recompute exists to drop).
    q, k, v: [B, h, T, d]."""
    scores = (q @ k.transpose(-2, -1)) / math.sqrt(q.shape[-1])
    t = scores.shape[-1]
    future = torch.ones(t, t, dtype=torch.bool, device=scores.device).triu(1)
    probs = F.softmax(scores.masked_fill(future, float("-inf")), dim=-1)
    return probs @ v


def causal_attention(qkv: torch.Tensor, n_head: int, head_dim: int, recompute_core: bool) -> torch.Tensor:
    b, t, _ = qkv.shape
    if native.active(qkv):
        from .flash import flash_attention

        return flash_attention(qkv, n_head, head_dim)
    y = qkv.view(b, t, n_head, 3, head_dim)
    q = y[:, :, :, 0].transpose(1, 2)
    k = y[:, :, :, 1].transpose(1, 2)
    v = y[:, :, :, 2].transpose(1, 2)
    out = recompute(core_attention, q, k, v) if recompute_core else core_attention(q, k, v)
    return out.transpose(1, 2).contiguous().view(b, t, n_head * head_dim)
