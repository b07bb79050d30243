"""Pipeline schedules (see :mod:`dstraining_b200.parallel.pipeline`)."""

from dstraining_b200.parallel.pipeline import Pipeline1F1B, PipelineInterleaved  # noqa: F401
