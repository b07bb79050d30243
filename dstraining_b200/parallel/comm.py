"""Autograd-aware tensor-parallel collectives (Megatron's conjugate pairs).

    copy_to_tp_region          f    fwd identity            bwd all-reduce
    reduce_from_tp_region      f̄    fwd all-reduce          bwd identity
    gather_from_tp_region           fwd all-gather(last)    bwd local slice
    gather_along_seq           g    fwd all-gather(seq)     bwd reduce-scatter(seq)
    reduce_scatter_along_seq   ḡ    fwd reduce-scatter(seq) bwd all-gather(seq)
    scatter_along_seq               fwd local seq slice     bwd all-gather(seq)

Same contract as the reference's ``dst/ops.py:159-192``. Activations are
``[batch, seq, hidden]`` (sequence is dim 1).

These standalone operators are the *unfused* path: they run on whatever
backend the group has (NCCL on GPUs, gloo on CPU). On CUDA bf16 the parallel
linear layers do not call them; they fuse the collective into their GEMM
kernels over NVLink peer memory (``dstraining_b200.ops.tp_fused``).

Gloo has no reduce-scatter: on gloo it is an all-to-all of the chunks
followed by a local sum in rank order (half the bytes of the reference's
all-reduce + slice emulation, ``dst/ops.py:102-118``); if the gloo build
lacks all-to-all, all-reduce + slice is used. This is the CPU path only.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from .topology import TPContext

SEQ_DIM = 1
_GLOO_A2A: dict = {}  # whether this gloo build supports all_to_all_single (probed on first use)


def _is_gloo(group) -> bool:
    try:
        return dist.get_backend(group) == "gloo"
    except Exception:  # pragma: no cover - uninitialised backends
        return False


def all_reduce_sum(t: torch.Tensor, tp: TPContext) -> torch.Tensor:
    """Out-of-place sum over the group (inputs of autograd functions and
    incoming gradients must not be mutated)."""
    out = t.contiguous().clone()
    dist.all_reduce(out, group=tp.group)
    return out


def all_gather_dim(t: torch.Tensor, tp: TPContext, dim: int) -> torch.Tensor:
    """Concatenate every rank's ``t`` along ``dim`` (group order); one collective."""
    t = t.contiguous()
    if dim == 0 and not _is_gloo(tp.group):
        out = torch.empty((t.shape[0] * tp.world, *t.shape[1:]), dtype=t.dtype, device=t.device)
        dist.all_gather_into_tensor(out, t, group=tp.group)
        return out
    # Gather along dim 0 of a moved view, then move back: one collective.
    moved = t.movedim(dim, 0).contiguous()
    if _is_gloo(tp.group):
        parts = [torch.empty_like(moved) for _ in range(tp.world)]
        dist.all_gather(parts, moved, group=tp.group)
        full = torch.cat(parts, dim=0)
    else:
        full = torch.empty((moved.shape[0] * tp.world, *moved.shape[1:]), dtype=t.dtype, device=t.device)
        dist.all_gather_into_tensor(full, moved, group=tp.group)
    return full.movedim(0, dim).contiguous()


def reduce_scatter_dim(t: torch.Tensor, tp: TPContext, dim: int) -> torch.Tensor:
    """Sum ``t`` over the group and keep this rank's equal slice along ``dim``."""
    n = t.shape[dim]
    if n % tp.world:
        raise ValueError(f"dim {dim} of size {n} not divisible by tp {tp.world}")
    chunk = n // tp.world
    if _is_gloo(tp.group):
        if _GLOO_A2A.get("ok", True):
            try:
                moved = t.movedim(dim, 0).contiguous()
                recv = torch.empty_like(moved)
                dist.all_to_all_single(recv, moved, group=tp.group)  # chunk j of recv comes from rank j
                _GLOO_A2A["ok"] = True
                out = recv.view(tp.world, chunk, *moved.shape[1:]).sum(0)  # fixed rank order
                return out.movedim(0, dim).contiguous()
            except RuntimeError:
                if "ok" in _GLOO_A2A:
                    raise  # worked before: a real failure, not a missing capability
                _GLOO_A2A["ok"] = False
        return all_reduce_sum(t, tp).narrow(dim, tp.rank * chunk, chunk).contiguous()
    moved = t.movedim(dim, 0).contiguous()
    out = torch.empty((chunk, *moved.shape[1:]), dtype=t.dtype, device=t.device)
    dist.reduce_scatter_tensor(out, moved, group=tp.group)
    return out.movedim(0, dim).contiguous()


def local_slice(t: torch.Tensor, tp: TPContext, dim: int) -> torch.Tensor:
    """This rank's equal slice of ``t`` along ``dim`` (no communication)."""
    chunk = t.shape[dim] // tp.world
    return t.narrow(dim, tp.rank * chunk, chunk).contiguous()


class _CopyToTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, tp):
        ctx.tp = tp
        return x

    @staticmethod
    def backward(ctx, g):
        return all_reduce_sum(g, ctx.tp), None


class _ReduceFromTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, tp):
        return all_reduce_sum(x, tp)

    @staticmethod
    def backward(ctx, g):
        return g, None


class _GatherLastDim(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, tp):
        ctx.tp = tp
        return all_gather_dim(x, tp, x.dim() - 1)

    @staticmethod
    def backward(ctx, g):
        return local_slice(g, ctx.tp, g.dim() - 1), None


class _GatherSeq(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, tp):
        ctx.tp = tp
        return all_gather_dim(x, tp, SEQ_DIM)

    @staticmethod
    def backward(ctx, g):
        return reduce_scatter_dim(g, ctx.tp, SEQ_DIM), None


class _ReduceScatterSeq(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, tp):
        ctx.tp = tp
        return reduce_scatter_dim(x, tp, SEQ_DIM)

    @staticmethod
    def backward(ctx, g):
        return all_gather_dim(g, ctx.tp, SEQ_DIM), None


class _ScatterSeq(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, tp):
        ctx.tp = tp
        return local_slice(x, tp, SEQ_DIM)

    @staticmethod
    def backward(ctx, g):
        return all_gather_dim(g, ctx.tp, SEQ_DIM), None


def copy_to_tp_region(x: torch.Tensor, tp: TPContext) -> torch.Tensor:
    """f: identity forward, all-reduce of the gradient backward (``dst/ops.py:177-180``)."""
    return _CopyToTP.apply(x, tp) if tp.enabled else x


def reduce_from_tp_region(x: torch.Tensor, tp: TPContext) -> torch.Tensor:
    """f̄: all-reduce forward, identity backward (``dst/ops.py:183-186``)."""
    return _ReduceFromTP.apply(x, tp) if tp.enabled else x


def gather_from_tp_region(x: torch.Tensor, tp: TPContext) -> torch.Tensor:
    """All-gather along the last dimension forward, local slice backward (``dst/ops.py:189-192``)."""
    return _GatherLastDim.apply(x, tp) if tp.enabled else x


def gather_along_seq(x: torch.Tensor, tp: TPContext) -> torch.Tensor:
    """g: all-gather along the sequence forward, reduce-scatter backward (``dst/ops.py:159-162``)."""
    return _GatherSeq.apply(x, tp) if tp.enabled else x


def reduce_scatter_along_seq(x: torch.Tensor, tp: TPContext) -> torch.Tensor:
    """ḡ: reduce-scatter along the sequence forward, all-gather backward (``dst/ops.py:165-168``)."""
    return _ReduceScatterSeq.apply(x, tp) if tp.enabled else x


def scatter_along_seq(x: torch.Tensor, tp: TPContext) -> torch.Tensor:
    """Local sequence slice forward, all-gather backward (``dst/ops.py:171-174``)."""
    return _ScatterSeq.apply(x, tp) if tp.enabled else x
