"""Tensor-parallel conjugate operators (see :mod:`dstraining_b200.parallel.comm`)."""

from dstraining_b200.parallel.comm import (  # noqa: F401
    SEQ_DIM,
    copy_to_tp_region,
    gather_along_seq,
    gather_from_tp_region,
    reduce_from_tp_region,
    reduce_scatter_along_seq,
    scatter_along_seq,
)
