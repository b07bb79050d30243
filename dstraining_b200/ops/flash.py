"""Autograd wrapper of the native causal flash attention (``csrc/attn_tc.cu``).

The tcgen05 kernels work on 128-row query and key tiles. A sequence length
that is not a multiple of 128 is zero-padded at the end up to the next one
and the padding sliced off again; under the causal mask this is exact:

* a real query row ``i < T`` only sees keys ``j <= i < T``, so the padded keys
  never enter its softmax, output or log-sum-exp;
* in backward the padded query rows get ``dO = 0``; their ``D = rowsum(dO * O)``
  is 0, so ``dP = dO V^T = 0`` and ``dS = P (dP - D) = 0``: they add exactly
  zero to every real key's dK and dV (their scores are 0, so P stays finite).

Replaces the reference's materialised ``core_attention``
(``dst/model.py:106-119``) on CUDA bf16 tensors.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from . import native

TILE = 128


def padded_length(t: int) -> int:
    """Sequence length the kernels run on: ``t`` rounded up to a multiple of 128."""
    return -(-t // TILE) * TILE


def _pad_rows(x: torch.Tensor, tp: int) -> torch.Tensor:
    t = x.shape[1]
    return x if t == tp else F.pad(x, (0, 0, 0, tp - t))


class _FlashFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, n_head, head_dim):
        t = qkv.shape[1]
        tp = padded_length(t)
        qkv_p = _pad_rows(qkv.contiguous(), tp)
        out, lse = native.lib().flash_attn_fwd_tc(qkv_p, n_head, head_dim)
        ctx.save_for_backward(qkv_p, out, lse)
        ctx.meta = (n_head, head_dim, t)
        return out if tp == t else out[:, :t].contiguous()

    @staticmethod
    def backward(ctx, dout):
        qkv_p, out, lse = ctx.saved_tensors
        n_head, head_dim, t = ctx.meta
        dout_p = _pad_rows(dout.contiguous(), qkv_p.shape[1])
        dqkv = native.lib().flash_attn_bwd_tc(dout_p, qkv_p, out, lse, n_head, head_dim)
        return (dqkv if dqkv.shape[1] == t else dqkv[:, :t].contiguous()), None, None


def flash_attention(qkv: torch.Tensor, n_head: int, head_dim: int) -> torch.Tensor:
    """qkv [B, T, n_head * 3 * head_dim] (head-major q|k|v) -> [B, T, n_head * head_dim]."""
    return _FlashFn.apply(qkv, n_head, head_dim)
