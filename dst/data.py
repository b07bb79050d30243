"""Token sources (see :mod:`dstraining_b200.utils.data`)."""

from dstraining_b200.utils.data import SyntheticShard, TokenShard  # noqa: F401
