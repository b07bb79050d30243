"""Vocab-parallel cross-entropy (PyTorch path) against ``F.cross_entropy`` on
the real vocabulary: loss and logit gradient, with padded columns that must
get zero gradient. Multi-rank shards are covered by the TP suites."""

import torch
import torch.nn.functional as F

from dstraining_b200.ops.cross_entropy import vocab_parallel_cross_entropy
from dstraining_b200.parallel.topology import SINGLE


def test_matches_cross_entropy_with_padding():
    g = torch.Generator().manual_seed(0)
    n, real, padded = 96, 250, 256
    logits = (torch.randn(n, padded, generator=g) * 3).requires_grad_(True)
    targets = torch.randint(0, real, (n,), generator=g)
    loss = vocab_parallel_cross_entropy(logits, targets, SINGLE, real)
    ref_in = logits.detach()[:, :real].clone().requires_grad_(True)
    ref = F.cross_entropy(ref_in, targets)
    torch.testing.assert_close(loss, ref, atol=1e-6, rtol=1e-6)
    loss.backward(torch.tensor(0.5))
    ref.backward(torch.tensor(0.5))
    torch.testing.assert_close(logits.grad[:, :real], ref_in.grad, atol=1e-7, rtol=1e-5)
    assert logits.grad[:, real:].abs().max().item() == 0


def test_bf16_logits_and_3d_shape():
    g = torch.Generator().manual_seed(1)
    logits = torch.randn(2, 8, 128, generator=g).to(torch.bfloat16).requires_grad_(True)
    targets = torch.randint(0, 100, (2, 8), generator=g)
    loss = vocab_parallel_cross_entropy(logits, targets, SINGLE, 100)
    ref = F.cross_entropy(logits.detach().float()[..., :100].reshape(-1, 100), targets.reshape(-1))
    torch.testing.assert_close(loss, ref, atol=1e-5, rtol=1e-5)
    loss.backward()
    assert logits.grad.dtype == torch.bfloat16 and logits.grad.shape == logits.shape
