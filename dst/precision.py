"""bf16 + fp32 master weights (see :mod:`dstraining_b200.optim.precision`)."""

from dstraining_b200.optim.precision import MasterWeightOptimizer  # noqa: F401
