"""Sequence lengths that are not a multiple of the attention kernels' 128-row
tiles are zero-padded by ``ops/flash.py``. Checked on the CPU with fp64
stand-ins for the two kernels (same signatures, same 128-multiple
requirement, same saved base-2 log-sum-exp): the padded forward and backward
equal causal attention on the unpadded sequence."""

import math

import pytest
import torch
import torch.nn.functional as F

from dstraining_b200.ops import flash, native


def _attn(qkv, H, D):
    B, T, _ = qkv.shape
    y = qkv.view(B, T, H, 3, D)
    q, k, v = (y[:, :, :, i].transpose(1, 2) for i in range(3))
    s = (q @ k.transpose(-2, -1)) / math.sqrt(D)
    s = s.masked_fill(torch.ones(T, T, dtype=torch.bool).triu(1), float("-inf"))
    lse2 = torch.logsumexp(s, -1) / math.log(2.0)
    o = F.softmax(s, -1) @ v
    return o.transpose(1, 2).reshape(B, T, H * D), lse2


class _FakeKernels:
    """Stand-ins for ``flash_attn_fwd_tc`` / ``flash_attn_bwd_tc``."""

    def __init__(self):
        self.lengths = []

    def flash_attn_fwd_tc(self, qkv, H, D, mode=0):
        assert qkv.is_contiguous() and qkv.shape[1] % 128 == 0
        self.lengths.append(qkv.shape[1])
        return _attn(qkv, H, D)

    def flash_attn_bwd_tc(self, dout, qkv, out, lse, H, D, mode=0):
        assert qkv.shape[1] % 128 == 0 and dout.shape == out.shape and lse.shape[-1] == qkv.shape[1]
        with torch.enable_grad():  # autograd runs backward functions with grad mode off
            x = qkv.detach().clone().requires_grad_(True)
            o, _ = _attn(x, H, D)
            o.backward(dout)
        return x.grad


@pytest.fixture
def fake(monkeypatch):
    k = _FakeKernels()
    monkeypatch.setattr(native, "_LIB", k)
    monkeypatch.setattr(native, "_DEBUG", None)
    monkeypatch.delenv("DST_DEBUG_SYNC", raising=False)
    return k


@pytest.mark.parametrize("T", [1, 72, 127, 128, 200, 300])
def test_padded_attention_equals_unpadded(fake, T):
    torch.manual_seed(T)
    B, H, D = 2, 3, 16
    qkv = torch.randn(B, T, 3 * H * D, dtype=torch.float64).requires_grad_(True)
    dout = torch.randn(B, T, H * D, dtype=torch.float64)
    out = flash.flash_attention(qkv, H, D)
    assert out.shape == (B, T, H * D) and out.is_contiguous()
    assert fake.lengths == [flash.padded_length(T)]
    out.backward(dout)
    ref_x = qkv.detach().clone().requires_grad_(True)
    ref, _ = _attn(ref_x, H, D)
    ref.backward(dout)
    torch.testing.assert_close(out, ref, rtol=1e-12, atol=1e-12)
    torch.testing.assert_close(qkv.grad, ref_x.grad, rtol=1e-10, atol=1e-12)


def test_padded_length():
    assert [flash.padded_length(t) for t in (1, 127, 128, 129, 1024, 1025)] == [128, 128, 128, 256, 1024, 1152]
