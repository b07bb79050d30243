"""Process grid, collectives, pipeline schedules and DP reduction."""

from .topology import (  # noqa: F401
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
