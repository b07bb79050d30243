"""Loader for the in-tree sm_100a extension (``dstraining_b200/_C*.so``).

Dispatch rule used by every op in this package: a CUDA bfloat16 tensor runs
the hand-written sm_100a kernels; anything else (CPU tensors, fp32 oracle
runs) runs plain PyTorch. There is no silent fallback on the GPU path: if a
CUDA bf16 op is requested and the extension did not load, :func:`lib` raises.
Set ``DST_NATIVE=0`` to force the PyTorch path everywhere (used only to A/B
against the oracle).

Debug mode (``DST_DEBUG_SYNC=1``): every call into the extension is followed
by a device synchronisation and a read of the per-device status word, so an
asynchronous CUDA error or a timed-out bounded wait is reported by the op
that caused it (:class:`NativeOpError` names it) instead of by some later
API call. This is the stand-in for a sanitizer run; it serialises the GPU
and is meant for debugging only.
"""

from __future__ import annotations

import importlib
import os

import torch

_LIB = None
_ERR = None
_DEBUG = None

# status codes written by the kernels' bounded waits (csrc/ptx.cuh)
STATUS_NAMES = {
    1: "timeout waiting for a TMA load",
    2: "timeout waiting for a free shared-memory stage",
    3: "timeout waiting for a TMEM accumulator",
    4: "timeout waiting for a free TMEM accumulator",
    5: "timeout waiting for a peer rank",
    6: "bad argument",
    7: "token or target id outside the vocabulary",
}


class NativeOpError(RuntimeError):
    """A native op left a CUDA error or a non-zero status word (debug mode)."""


class _Checked:
    """Proxy over the extension module: calls pass through, then the device
    is synchronised and the status word read (and cleared)."""

    _SKIP = {"read_status", "num_sms", "status_ptr"}

    def __init__(self, mod):
        self._mod = mod

    def __getattr__(self, name):
        attr = getattr(self._mod, name)
        if not callable(attr) or name in self._SKIP:
            return attr

        def call(*args, **kwargs):
            out = attr(*args, **kwargs)
            try:
                torch.cuda.synchronize()
            except Exception as e:  # noqa: BLE001 - re-raised with the op name
                raise NativeOpError(f"native op {name!r} left a CUDA error: {e}") from e
            code = int(self._mod.read_status(True))
            if code:
                raise NativeOpError(f"native op {name!r} reported status {code} "
                                    f"({STATUS_NAMES.get(code, 'unknown')})")
            return out

        return call


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


def debug_sync() -> bool:
    return os.environ.get("DST_DEBUG_SYNC", "0") not in ("", "0")


def lib():
    """The extension module; raises with the import error if it is missing.
    Under ``DST_DEBUG_SYNC=1`` a checking proxy of it (see the module doc)."""
    global _DEBUG
    _load()
    if _LIB is None:
        raise RuntimeError(
            "dstraining_b200 native extension is not built or failed to load "
            f"({_ERR!r}); run `python setup.py build_ext --inplace`"
        )
    if debug_sync():
        if _DEBUG is None:
            _DEBUG = _Checked(_LIB)
        return _DEBUG
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
