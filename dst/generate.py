"""Sampling from a trained model (new; the reference has none). See
:mod:`dstraining_b200.utils.generate`."""

from dstraining_b200.utils.generate import generate, load_model  # noqa: F401
