"""Data-parallel gradient reduction (see :mod:`dstraining_b200.parallel.dp`)."""

from dstraining_b200.parallel.dp import GradReducer, allreduce_gradients  # noqa: F401
