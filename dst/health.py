"""Failure detection for multi-rank training (new; the reference has none).
See :mod:`dstraining_b200.parallel.health`."""

from dstraining_b200.parallel.health import (  # noqa: F401
    Heartbeat,
    PeerFailure,
    StepGate,
    Watchdog,
    report_failure,
    stale_ranks,
    start_monitoring,
)
