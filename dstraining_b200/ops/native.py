"""Loader for the in-tree sm_100a extension (``dstraining_b200/_C*.so``).

Dispatch rule used by every op in this package: a CUDA bfloat16 tensor runs
the hand-written sm_100a kernels; anything else (CPU tensors, fp32 oracle
runs) runs plain PyTorch. There is no silent fallback on the GPU path: if a
CUDA bf16 op is requested and the extension did not load, :func:`lib` raises.
Set ``DST_NATIVE=0`` to force the PyTorch path everywhere (used only to A/B
against the oracle).
"""

from __future__ import annotations

import importlib
import os

import torch

_LIB = None
_ERR = None


def _load():
    global _LIB, _ERR
    if _LIB is not None or _ERR is not None:
        return
    try:
        _LIB = importlib.import_module("dstraining_b200._C")
    except Exception as e:  # noqa: BLE001 - surfaced verbatim by lib()
        _ERR = e


def available() -> bool:
    _load()
    return _LIB is not None


def lib():
    """The extension module; raises with the import error if it is missing."""
    _load()
    if _LIB is None:
        raise RuntimeError(
            "dstraining_b200 native extension is not built or failed to load "
            f"({_ERR!r}); run `python setup.py build_ext --inplace`"
        )
    return _LIB


def enabled() -> bool:
    return os.environ.get("DST_NATIVE", "1") != "0"


def active(*tensors: torch.Tensor) -> bool:
    """True when these tensors take the native path: all on CUDA, bf16."""
    if not enabled():
        return False
    for t in tensors:
        if t is None:
            continue
        if not (t.is_cuda and t.dtype == torch.bfloat16):
            return False
    return True
