"""Vocab-parallel cross-entropy (see :mod:`dstraining_b200.ops.cross_entropy`)."""

from dstraining_b200.ops.cross_entropy import vocab_parallel_cross_entropy  # noqa: F401
