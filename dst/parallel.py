"""Process grid and contexts (see :mod:`dstraining_b200.parallel.topology`)."""

from dstraining_b200.parallel.topology import (  # noqa: F401
    DP_SINGLE,
    PP_SINGLE,
    SINGLE,
    DPContext,
    PPContext,
    TPContext,
    default_device,
    init_distributed,
    make_topology,
    make_tp_context,
)
