"""Optional NVTX ranges for timeline tools (``DST_NVTX=1``).

``nvtx_range(name)`` is a context manager that pushes an NVTX range around
its body when ``DST_NVTX`` is set and CUDA is available, and does nothing
otherwise (no cost on the normal path). The trainer marks its phases
(``forward_backward``, ``dp_reduce``, ``finalize_grads``, ``optimizer``) and
the models mark each block, so a profiler timeline shows where a step's
time goes. The reference has no tracing (its only timing is a cumulative
wall-clock average in ``train.py:123-152``).
"""

from __future__ import annotations

import contextlib
import os

import torch


def enabled() -> bool:
    return os.environ.get("DST_NVTX", "0") not in ("", "0") and torch.cuda.is_available()


@contextlib.contextmanager
def nvtx_range(name: str):
    if not enabled():
        yield
        return
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()
