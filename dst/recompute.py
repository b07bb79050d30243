"""Selective recompute (see :mod:`dstraining_b200.ops.recompute`)."""

from dstraining_b200.ops.recompute import _Recompute, recompute  # noqa: F401
