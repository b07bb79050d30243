"""Optimizers."""

from .precision import MasterWeightOptimizer  # noqa: F401
