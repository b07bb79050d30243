"""Autograd wrapper of the native causal flash attention (``csrc/attn.cu``)."""

from __future__ import annotations

import torch

from . import native


class _FlashFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, n_head, head_dim):
        qkv = qkv.contiguous()
        lib = native.lib()
        # tcgen05 kernel for 128-multiple sequence lengths, mma.sync tiles otherwise;
        # both save the same base-2 log-sum-exp for the backward kernels.
        fwd = lib.flash_attn_fwd_tc if qkv.shape[1] % 128 == 0 else lib.flash_attn_fwd
        out, lse = fwd(qkv, n_head, head_dim)
        ctx.save_for_backward(qkv, out, lse)
        ctx.meta = (n_head, head_dim)
        return out

    @staticmethod
    def backward(ctx, dout):
        qkv, out, lse = ctx.saved_tensors
        n_head, head_dim = ctx.meta
        lib = native.lib()
        bwd = lib.flash_attn_bwd_tc if qkv.shape[1] % 128 == 0 else lib.flash_attn_bwd
        dqkv = bwd(dout.contiguous(), qkv, out, lse, n_head, head_dim)
        return dqkv, None, None


def flash_attention(qkv: torch.Tensor, n_head: int, head_dim: int) -> torch.Tensor:
    """qkv [B, T, n_head * 3 * head_dim] (head-major q|k|v) -> [B, T, n_head * head_dim]."""
    return _FlashFn.apply(qkv, n_head, head_dim)
