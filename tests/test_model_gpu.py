"""End-to-end native bf16 model vs the fp32 PyTorch model with identical
weights: loss and gradients agree to bf16 accuracy, training with
MasterWeightOptimizer makes the loss fall, and the native kernels (not a
PyTorch fallback) are what ran."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _cfg(**kw):
    from dstraining_b200.models.gpt import GPTConfig

    base = dict(vocab_size=1000, block_size=256, n_layer=2, n_head=4, n_embd=256, vocab_parallel_loss=True)
    base.update(kw)
    return GPTConfig(**base)


@pytest.mark.parametrize("head_dim", [64, 128])
def test_native_model_matches_fp32(cuda, head_dim):
    from dstraining_b200.models.gpt import GPT
    from dstraining_b200.ops import native
    from dstraining_b200.parallel.topology import SINGLE

    assert native.available(), "native extension must load on a GPU box"
    cfg = _cfg(n_head=256 // head_dim)
    m16 = GPT(cfg, SINGLE, seed=3).to(cuda).to(torch.bfloat16)
    m32 = GPT(cfg, SINGLE, seed=3).to(cuda)
    with torch.no_grad():
        for p16, p32 in zip(m16.parameters(), m32.parameters()):
            p32.copy_(p16.float())  # identical (bf16-representable) weights
    g = torch.Generator().manual_seed(0)
    idx = torch.randint(0, cfg.vocab_size, (4, cfg.block_size), generator=g).to(cuda)
    tgt = torch.randint(0, cfg.vocab_size, (4, cfg.block_size), generator=g).to(cuda)
    _, l16 = m16(idx, tgt)
    _, l32 = m32(idx, tgt)
    assert abs(l16.item() - l32.item()) < 2e-2
    l16.backward()
    l32.backward()
    worst = 0.0
    for (n, p16), p32 in zip(m16.named_parameters(), m32.parameters()):
        rel = ((p16.grad.float() - p32.grad).abs().max() / p32.grad.abs().max().clamp_min(1e-8)).item()
        worst = max(worst, rel)
        assert rel < 6e-2, n
    assert native.lib().read_status(True) == 0


def test_native_training_loss_falls(cuda):
    from dstraining_b200.models.gpt import GPT
    from dstraining_b200.optim.precision import MasterWeightOptimizer
    from dstraining_b200.parallel.topology import SINGLE

    cfg = _cfg()
    model = GPT(cfg, SINGLE, seed=1).to(cuda).to(torch.bfloat16)
    opt = MasterWeightOptimizer(model.parameters(), lr=1e-3)
    g = torch.Generator().manual_seed(0)
    idx = torch.randint(0, cfg.vocab_size, (4, cfg.block_size), generator=g).to(cuda)
    tgt = torch.randint(0, cfg.vocab_size, (4, cfg.block_size), generator=g).to(cuda)
    losses = []
    for _ in range(30):
        opt.zero_grad()
        _, loss = model(idx, tgt)
        loss.backward()
        opt.step()
        losses.append(loss.item())
    assert losses[-1] < losses[0] - 1.0, losses
