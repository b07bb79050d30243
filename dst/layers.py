"""Tensor-parallel linear layers (see :mod:`dstraining_b200.models.layers`)."""

from dstraining_b200.models.layers import ColumnParallelLinear, RowParallelLinear  # noqa: F401
