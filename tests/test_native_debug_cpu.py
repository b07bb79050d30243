"""Debug mode of the native-op loader (``DST_DEBUG_SYNC=1``), checked with a
fake extension module on the CPU: each call is followed by a synchronisation
and a status-word read, and a non-zero status raises an error naming the op."""

import pytest
import torch

from dstraining_b200.ops import native


class _FakeLib:
    def __init__(self):
        self.codes = []
        self.calls = []
        self.version = 3

    def read_status(self, clear=True):
        return self.codes.pop(0) if self.codes else 0

    def gemm(self, *args):
        self.calls.append(("gemm", args))
        return "out"

    def fused_dp_adam(self, *args):
        self.calls.append(("fused_dp_adam", args))


@pytest.fixture
def fake(monkeypatch):
    lib = _FakeLib()
    monkeypatch.setattr(native, "_LIB", lib)
    monkeypatch.setattr(native, "_DEBUG", None)
    monkeypatch.setattr(torch.cuda, "synchronize", lambda *a, **k: None)
    return lib


def test_plain_mode_returns_module(fake, monkeypatch):
    monkeypatch.delenv("DST_DEBUG_SYNC", raising=False)
    assert native.lib() is fake


def test_debug_mode_checks_every_call(fake, monkeypatch):
    monkeypatch.setenv("DST_DEBUG_SYNC", "1")
    lib = native.lib()
    assert lib is not fake
    assert lib.gemm(1, 2) == "out" and fake.calls == [("gemm", (1, 2))]
    assert lib.version == 3  # non-callables pass through
    fake.codes = [5]
    with pytest.raises(native.NativeOpError, match="fused_dp_adam.*status 5.*peer"):
        lib.fused_dp_adam(0)
    assert lib.read_status(True) == 0  # not wrapped


def test_debug_mode_reports_cuda_errors(fake, monkeypatch):
    monkeypatch.setenv("DST_DEBUG_SYNC", "1")

    def boom():
        raise RuntimeError("CUDA error: an illegal memory access was encountered")

    monkeypatch.setattr(torch.cuda, "synchronize", boom)
    with pytest.raises(native.NativeOpError, match="'gemm' left a CUDA error"):
        native.lib().gemm()
