"""Native (CUDA bf16) paths of the parallel linear layers.

Every GEMM runs on the tcgen05 kernel with its epilogue fused: bias,
GELU-tanh (also writing the pre-activation that backward needs), residual
add, and dGELU in the backward GEMM that produces the MLP hidden gradient.
The MLP is one autograd function so that dGELU can live in the c_proj
backward epilogue instead of a separate pass.

Tensor parallelism: with tp > 1 the column layer's entry collective (g
all-gather along the sequence, or f) and the row layer's exit collective
(ḡ reduce-scatter or f̄ all-reduce) run through
:mod:`dstraining_b200.ops.tp_fused`, whose kernels overlap the NVLink
transfer with the GEMM tiles; the unfused NCCL versions in
:mod:`dstraining_b200.parallel.comm` remain the oracle.
"""

from __future__ import annotations

import os

from typing import Optional

import torch

from ..parallel.comm import all_gather_dim, all_reduce_sum, reduce_scatter_dim
from ..parallel.topology import TPContext
from . import tp_fused
from .gemm import EPI_BIAS, EPI_BIAS_GELU, EPI_BIAS_RESID, EPI_DGELU, EPI_STORE, bias_grad, gemm, weight_grad

SEQ = 1


def _enter(x: torch.Tensor, tp: TPContext, mode: str) -> torch.Tensor:
    """Forward of the column layer's entry operator (g or f)."""
    if tp.enabled and mode == "sequence":
        return all_gather_dim(x, tp, SEQ)
    return x


def _enter_bwd(dx: torch.Tensor, tp: TPContext, mode: str) -> torch.Tensor:
    if not tp.enabled:
        return dx
    if mode == "sequence":
        return reduce_scatter_dim(dx, tp, SEQ)
    return all_reduce_sum(dx, tp)


def _exit(y: torch.Tensor, tp: TPContext, mode: str) -> torch.Tensor:
    """Forward of the row layer's exit operator (ḡ or f̄)."""
    if not tp.enabled:
        return y
    if mode == "sequence":
        return reduce_scatter_dim(y, tp, SEQ)
    return all_reduce_sum(y, tp)


def _exit_bwd(dy: torch.Tensor, tp: TPContext, mode: str) -> torch.Tensor:
    if tp.enabled and mode == "sequence":
        return all_gather_dim(dy, tp, SEQ)
    return dy


def _flat(t: torch.Tensor) -> torch.Tensor:
    return t.reshape(-1, t.shape[-1])


class _ColumnFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, tp, mode, gelu):
        xf = _enter(x, tp, mode).contiguous()
        x2 = _flat(xf)
        if gelu:
            pre = torch.empty((x2.shape[0], w.shape[0]), dtype=x.dtype, device=x.device)
            y = gemm(x2, False, w, False, EPI_BIAS_GELU, bias=b, aux_out=pre)
            ctx.save_for_backward(x2, w, pre)
        else:
            y = gemm(x2, False, w, False, EPI_BIAS if b is not None else EPI_STORE, bias=b)
            ctx.save_for_backward(x2, w)
        ctx.meta = (tp, mode, gelu, b is not None, xf.shape)
        return y.view(*xf.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):
        tp, mode, gelu, has_bias, xshape = ctx.meta
        dy2 = _flat(dy).contiguous()
        if gelu:
            x2, w, pre = ctx.saved_tensors
            # Standalone GELU column layer: dGELU as a separate elementwise step.
            xp = pre.float()
            k0, k1 = 0.7978845608028654, 0.044715
            t = torch.tanh(k0 * (xp + k1 * xp**3))
            dgelu = 0.5 * (1 + t) + 0.5 * xp * (1 - t * t) * k0 * (1 + 3 * k1 * xp * xp)
            dy2 = (dy2.float() * dgelu).to(dy2.dtype)
        else:
            x2, w = ctx.saved_tensors
        dx = gemm(dy2, False, w, True, EPI_STORE).view(xshape)
        dw = weight_grad(dy2, x2)
        db = bias_grad(dy2) if has_bias else None
        return _enter_bwd(dx, tp, mode), dw, db, None, None, None


class _RowFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, residual, tp, mode):
        x2 = _flat(x.contiguous())
        ctx.save_for_backward(x2, w)
        ctx.meta = (tp, mode, b is not None, residual is not None, x.shape)
        if not tp.enabled:
            if residual is not None:
                r2 = _flat(residual.contiguous())
                y = gemm(x2, False, w, False, EPI_BIAS_RESID, bias=b, aux=r2)
            else:
                y = gemm(x2, False, w, False, EPI_BIAS if b is not None else EPI_STORE, bias=b)
            return y.view(*x.shape[:-1], w.shape[0])
        y = gemm(x2, False, w, False, EPI_STORE).view(*x.shape[:-1], w.shape[0])
        y = _exit(y, tp, mode)
        if b is not None:
            y = y + b
        if residual is not None:
            y = residual + y
        return y

    @staticmethod
    def backward(ctx, dy):
        x2, w = ctx.saved_tensors
        tp, mode, has_bias, has_res, xshape = ctx.meta
        dres = dy if has_res else None
        db = bias_grad(_flat(dy).contiguous()) if has_bias else None
        if tp.enabled and mode == "sequence" and has_bias:
            pass  # partial over the sequence shard; summed over TP by finalize_grads
        dyf = _exit_bwd(dy, tp, mode).contiguous()
        dy2 = _flat(dyf)
        dx = gemm(dy2, False, w, True, EPI_STORE).view(xshape)
        dw = weight_grad(dy2, x2)
        return dx, dw, db, dres, None, None


class _MLPFn(torch.autograd.Function):
    """c_proj(gelu(c_fc(x))) + residual with dGELU fused into the c_proj
    backward GEMM."""

    @staticmethod
    def forward(ctx, x, w1, b1, w2, b2, residual, tp, in_mode, out_mode):
        xf = _enter(x, tp, in_mode).contiguous()
        x2 = _flat(xf)
        pre = torch.empty((x2.shape[0], w1.shape[0]), dtype=x.dtype, device=x.device)
        h = gemm(x2, False, w1, False, EPI_BIAS_GELU, bias=b1, aux_out=pre)
        if not tp.enabled:
            if residual is not None:
                y = gemm(h, False, w2, False, EPI_BIAS_RESID, bias=b2, aux=_flat(residual.contiguous()))
            else:
                y = gemm(h, False, w2, False, EPI_BIAS if b2 is not None else EPI_STORE, bias=b2)
            y = y.view(*x.shape[:-1], w2.shape[0])
        else:
            y = gemm(h, False, w2, False, EPI_STORE).view(*xf.shape[:-1], w2.shape[0])
            y = _exit(y, tp, out_mode)
            if b2 is not None:
                y = y + b2
            if residual is not None:
                y = residual + y
        ctx.save_for_backward(x2, w1, pre, h, w2)
        ctx.meta = (tp, in_mode, out_mode, b1 is not None, b2 is not None, residual is not None, xf.shape)
        return y

    @staticmethod
    def backward(ctx, dy):
        x2, w1, pre, h, w2 = ctx.saved_tensors
        tp, in_mode, out_mode, has_b1, has_b2, has_res, xshape = ctx.meta
        dres = dy if has_res else None
        db2 = bias_grad(_flat(dy).contiguous()) if has_b2 else None
        dyf = _exit_bwd(dy, tp, out_mode).contiguous()
        dy2 = _flat(dyf)
        dpre = gemm(dy2, False, w2, True, EPI_DGELU, aux=pre)
        dw2 = weight_grad(dy2, h)
        dx = gemm(dpre, False, w1, True, EPI_STORE).view(xshape)
        dw1 = weight_grad(dpre, x2)
        db1 = bias_grad(dpre) if has_b1 else None
        return _enter_bwd(dx, tp, in_mode), dw1, db1, dw2, db2, dres, None, None, None


def _seq_len(x: torch.Tensor, tp: TPContext, sharded: bool) -> int:
    return x.shape[1] * tp.world if sharded else x.shape[1]


def column_parallel_linear(x, w, b, tp: TPContext, mode: str, activation: Optional[str]):
    if activation is None and x.dim() == 3 and tp_fused.usable(tp, _seq_len(x, tp, mode == "sequence")):
        return tp_fused.column_parallel(x, w, b, tp, mode)
    return _ColumnFn.apply(x, w, b, tp, mode, activation == "gelu_tanh")


def row_parallel_linear(x, w, b, tp: TPContext, mode: str, residual: Optional[torch.Tensor]):
    if x.dim() == 3 and tp_fused.usable(tp, x.shape[1]):
        return tp_fused.row_parallel(x, w, b, residual, tp, mode)
    return _RowFn.apply(x, w, b, residual, tp, mode)


def mlp(x, c_fc, c_proj, residual: Optional[torch.Tensor]):
    tp = c_fc.tp
    if (
        c_fc.input_mode == "sequence"
        and c_proj.output_mode == "sequence"
        and x.dim() == 3
        and tp_fused.usable(tp, x.shape[1] * tp.world)
    ):
        return tp_fused.mlp_sequence_parallel(x, c_fc.weight, c_fc.bias, c_proj.weight, c_proj.bias, residual, tp)
    if (
        os.environ.get("DST_FUSED_TP_MLP", "1") != "0"  # 0: NCCL all-reduces around the native GEMMs
        and c_fc.input_mode == "replicated"
        and c_proj.output_mode == "replicated"
        and x.dim() == 3
        and tp_fused.usable(tp, x.shape[1])
    ):
        return tp_fused.mlp_replicated(x, c_fc.weight, c_fc.bias, c_proj.weight, c_proj.bias, residual, tp)
    return _MLPFn.apply(
        x, c_fc.weight, c_fc.bias, c_proj.weight, c_proj.bias, residual, c_fc.tp, c_fc.input_mode, c_proj.output_mode
    )
