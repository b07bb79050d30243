"""Sharded, reshardable checkpoints (new; the reference has none). See
:mod:`dstraining_b200.utils.checkpoint`."""

from dstraining_b200.utils.checkpoint import PendingSave, inspect, latest, load, save, verify_shard  # noqa: F401
