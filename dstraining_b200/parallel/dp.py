"""Data-parallel gradient reduction.

``allreduce_gradients``: one blocking all-reduce per parameter, then divide
by the DP size - the simple baseline (``dst/dp.py:43-49``).

``GradReducer``: bucketed and overlapped with backward. Parameters are taken
in reverse registration order (roughly the order backward finishes them) and
packed into buckets of at least ``bucket_bytes`` (default 25 MiB). Each bucket
owns ONE persistent flat buffer for its whole life. A post-accumulate-grad
hook copies a finished gradient into its slot (so the copy runs on the
compute stream right after the gradient is produced, instead of as one
flatten pass later); when the last slot of a bucket fills, the bucket's
all-reduce is launched asynchronously and overlaps the rest of backward.
``finish()`` waits, scales by ``1/dp`` and points each ``param.grad`` at its
slot of the reduced buffer - there is no unflatten copy.

For pipeline schedules, whose backward runs many times per step, construct
with ``overlap=False`` and call ``reduce()`` after ``train_step``.

On CUDA bf16 with the native extension and a multi-GPU DP group, use
:class:`dstraining_b200.optim.fused_dp.FusedDPAdam` instead: it reduces each
bucket over NVLink peer memory and applies the fp32-master Adam update in
the same kernel.
"""

from __future__ import annotations

from typing import Dict, List

import torch
import torch.distributed as dist
import torch.nn as nn

from .topology import DPContext


def allreduce_gradients(module: nn.Module, dp: DPContext) -> None:
    """Naive DP: one blocking all-reduce per gradient, then divide by the world (``dst/dp.py:43-49``)."""
    if not dp.enabled:
        return
    for p in module.parameters():
        if p.grad is not None:
            dist.all_reduce(p.grad, group=dp.group)
            p.grad /= dp.world


def build_buckets(params: List[nn.Parameter], bucket_bytes: int) -> List[List[nn.Parameter]]:
    """Greedy packing in the given order; a bucket closes once it reaches
    ``bucket_bytes`` (so one huge tensor gets a bucket of its own)."""
    out, cur, size = [], [], 0
    for p in params:
        cur.append(p)
        size += p.numel() * p.element_size()
        if size >= bucket_bytes:
            out.append(cur)
            cur, size = [], 0
    if cur:
        out.append(cur)
    return out


class _Bucket:
    def __init__(self, params: List[nn.Parameter]):
        self.params = params
        p0 = params[0]
        self.offsets = []
        off = 0
        for p in params:
            self.offsets.append(off)
            off += p.numel()
        self.flat = torch.zeros(off, dtype=p0.dtype, device=p0.device)
        self.filled = set()
        self.work = None

    def slot(self, i: int) -> torch.Tensor:
        p = self.params[i]
        return self.flat[self.offsets[i] : self.offsets[i] + p.numel()].view_as(p)

    def stage(self, i: int) -> None:
        g = self.params[i].grad
        if g is None:
            self.slot(i).zero_()
        elif g.data_ptr() != self.slot(i).data_ptr():
            self.slot(i).copy_(g)

    def launch(self, dp: DPContext) -> None:
        for i in range(len(self.params)):
            if i not in self.filled:
                self.stage(i)
        self.work = dist.all_reduce(self.flat, group=dp.group, async_op=True)

    def finish(self, dp: DPContext) -> None:
        self.work.wait()
        self.flat.div_(dp.world)
        for i, p in enumerate(self.params):
            if p.grad is not None:
                p.grad = self.slot(i)
        self.work = None
        self.filled = set()


class GradReducer:
    """Bucketed, overlapped DP gradient averaging (``dst/dp.py:78-142``): parameters in
    reverse order are packed into persistent flat buckets (~``bucket_bytes``); with
    ``overlap`` a post-accumulate-grad hook launches a bucket's all-reduce as soon as
    all its gradients exist; ``finish()`` waits, averages and exposes the buffers
    as ``param.grad``. ``reduce()`` launches every bucket (pipeline path); ``defer``
    silences the hooks while gradients are being accumulated."""

    def __init__(self, module: nn.Module, dp: DPContext, *, bucket_bytes: int = 25 * 1024 * 1024, overlap: bool = True):
        self.dp = dp
        self.overlap = overlap and dp.enabled
        self.defer = False  # set while accumulating gradients over micro-batches
        self.buckets: List[_Bucket] = []
        self._where: Dict[int, tuple] = {}
        if not dp.enabled:
            return
        params = [p for p in module.parameters() if p.requires_grad][::-1]
        for group in build_buckets(params, bucket_bytes):
            b = _Bucket(group)
            for i, p in enumerate(group):
                self._where[id(p)] = (b, i)
            self.buckets.append(b)
        if self.overlap:
            for p in params:
                p.register_post_accumulate_grad_hook(self._hook)

    def _hook(self, p: nn.Parameter) -> None:
        if self.defer:
            return  # gradient accumulation: only the last micro-batch's backward reduces
        b, i = self._where[id(p)]
        b.stage(i)
        b.filled.add(i)
        if len(b.filled) == len(b.params) and b.work is None:
            b.launch(self.dp)

    def reduce(self) -> None:
        """Launch every bucket's all-reduce back to back (pipeline path)."""
        if not self.dp.enabled:
            return
        for b in self.buckets:
            if b.work is None:
                b.launch(self.dp)

    def finish(self) -> None:
        """Wait for the reductions, average, and expose the reduced buffers
        as ``param.grad``."""
        if not self.dp.enabled:
            return
        for b in self.buckets:
            if b.work is None:
                b.launch(self.dp)  # a bucket backward never completed: still reduce
            b.finish(self.dp)
