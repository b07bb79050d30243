"""Tensor-parallel linear layers.

Both layers draw the FULL ``[out, in]`` weight from the caller's seeded
generator (``normal(0, init_std)``) and keep their shard, so a model built at
any TP degree holds exact slices of the weights the tp=1 model holds. That
decomposition-invariant init is a public contract (the reference,
``dst/layers.py:64-67,116-119``): checkpoints reshard by slicing and every
correctness test compares against a single-process model without copying
weights.

``ColumnParallelLinear``: ``Y = X A`` with ``A`` split by output columns (a
row split of torch's ``[out, in]`` weight). Entry operator: ``f`` (input
replicated) or ``g`` (input sequence-sharded, all-gathered). Optional fused
activation (GELU-tanh) and optional ``gather_output``.

``RowParallelLinear``: ``Z = sum_r Y_r B_r`` with ``B`` split by input rows.
Exit operator: ``f̄`` (all-reduce) or ``ḡ`` (reduce-scatter along the
sequence); the full bias is added after the reduction, then an optional
residual. Under sequence parallelism the bias sees only this rank's sequence
chunk in backward, so it is tagged ``sequence_parallel_replicated``.

On CUDA bf16 the collective and the GEMM run as one native kernel
(:mod:`dstraining_b200.ops.linear`); elsewhere the unfused PyTorch path
below is the oracle.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..ops import native
from ..parallel.comm import (
    copy_to_tp_region,
    gather_along_seq,
    gather_from_tp_region,
    reduce_from_tp_region,
    reduce_scatter_along_seq,
)
from ..parallel.topology import TPContext

ACTIVATIONS = (None, "gelu_tanh")


def _draw_full(out_features: int, in_features: int, std: float, generator) -> torch.Tensor:
    w = torch.empty(out_features, in_features)
    w.normal_(0.0, std, generator=generator)
    return w


class ColumnParallelLinear(nn.Module):
    """Linear layer whose output features are split over TP (``dst/layers.py:26-78``):
    the full ``[out, in]`` weight is drawn from the caller's generator and the
    row shard kept; input ``"replicated"`` (f) or ``"sequence"`` (g); optional
    ``gather_output``; CUDA bf16 runs the fused NVLink GEMMs."""

    def __init__(
        self,
        in_features: int,
        out_features: int,
        tp: TPContext,
        *,
        bias: bool = True,
        gather_output: bool = False,
        input_mode: str = "replicated",
        init_std: float = 0.02,
        generator: Optional[torch.Generator] = None,
    ):
        super().__init__()
        if out_features % tp.world:
            raise ValueError(f"out_features {out_features} not divisible by tp {tp.world}")
        if input_mode not in ("replicated", "sequence"):
            raise ValueError(f"input_mode must be 'replicated' or 'sequence', got {input_mode!r}")
        self.tp = tp
        self.in_features = in_features
        self.out_features = out_features
        self.gather_output = gather_output
        self.input_mode = input_mode
        rows = out_features // tp.world
        full = _draw_full(out_features, in_features, init_std, generator)
        self.weight = nn.Parameter(full[tp.rank * rows : (tp.rank + 1) * rows].clone())
        self.bias = nn.Parameter(torch.zeros(rows)) if bias else None

    def forward(self, x: torch.Tensor, activation: Optional[str] = None) -> torch.Tensor:
        assert activation in ACTIVATIONS
        if native.active(x, self.weight):
            from ..ops.linear import column_parallel_linear

            y = column_parallel_linear(x, self.weight, self.bias, self.tp, self.input_mode, activation)
            return gather_from_tp_region(y, self.tp) if self.gather_output else y
        if self.input_mode == "sequence":
            x = gather_along_seq(x, self.tp)
        else:
            x = copy_to_tp_region(x, self.tp)
        y = F.linear(x, self.weight, self.bias)
        if activation == "gelu_tanh":
            y = F.gelu(y, approximate="tanh")
        if self.gather_output:
            y = gather_from_tp_region(y, self.tp)
        return y


class RowParallelLinear(nn.Module):
    """Linear layer whose input features are split over TP (``dst/layers.py:81-135``):
    the column shard of the full weight is kept; output all-reduced (f̄) or
    reduce-scattered along the sequence (ḡ), then the full bias (and an optional
    residual) added."""

    def __init__(
        self,
        in_features: int,
        out_features: int,
        tp: TPContext,
        *,
        bias: bool = True,
        output_mode: str = "replicated",
        init_std: float = 0.02,
        generator: Optional[torch.Generator] = None,
    ):
        super().__init__()
        if in_features % tp.world:
            raise ValueError(f"in_features {in_features} not divisible by tp {tp.world}")
        if output_mode not in ("replicated", "sequence"):
            raise ValueError(f"output_mode must be 'replicated' or 'sequence', got {output_mode!r}")
        self.tp = tp
        self.in_features = in_features
        self.out_features = out_features
        self.output_mode = output_mode
        cols = in_features // tp.world
        full = _draw_full(out_features, in_features, init_std, generator)
        self.weight = nn.Parameter(full[:, tp.rank * cols : (tp.rank + 1) * cols].clone())
        self.bias = nn.Parameter(torch.zeros(out_features)) if bias else None
        if self.bias is not None and output_mode == "sequence":
            self.bias.sequence_parallel_replicated = True

    def forward(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        if native.active(x, self.weight):
            from ..ops.linear import row_parallel_linear

            return row_parallel_linear(x, self.weight, self.bias, self.tp, self.output_mode, residual)
        y = F.linear(x, self.weight)
        if self.output_mode == "sequence":
            y = reduce_scatter_along_seq(y, self.tp)
        else:
            y = reduce_from_tp_region(y, self.tp)
        if self.bias is not None:
            y = y + self.bias
        if residual is not None:
            y = residual + y
        return y
