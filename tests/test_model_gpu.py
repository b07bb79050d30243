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


def test_block_recompute_native(cuda):
    """Full-block recompute (``GPTConfig.recompute_blocks``) on the native bf16
    path: each block keeps only its input and runs again in backward; loss
    and gradients equal those of the run that stores every activation."""
    from dstraining_b200.models.gpt import GPT
    from dstraining_b200.ops import native
    from dstraining_b200.parallel.topology import SINGLE

    runs = []
    for full in (False, True):
        cfg = _cfg(recompute_blocks=full)
        m = GPT(cfg, SINGLE, seed=4).to(cuda).to(torch.bfloat16)
        g = torch.Generator().manual_seed(1)
        idx = torch.randint(0, cfg.vocab_size, (4, cfg.block_size), generator=g).to(cuda)
        tgt = torch.randint(0, cfg.vocab_size, (4, cfg.block_size), generator=g).to(cuda)
        _, loss = m(idx, tgt)
        loss.backward()
        runs.append((loss.item(), [(n, p.grad.float()) for n, p in m.named_parameters()]))
    (l0, g0), (l1, g1) = runs
    assert abs(l0 - l1) < 1e-4
    for (n, a), (_, b) in zip(g0, g1):
        assert ((a - b).abs().max() / a.abs().max().clamp_min(1e-8)).item() < 1e-2, n
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


def test_trainer_checkpoint_resume_gpu(cuda, monkeypatch, tmp_path):
    """Trainer on CUDA bf16 (bucketed fused Adam): training 6 steps straight
    equals 3 steps + sharded checkpoint + fresh trainer + load + 3 steps."""
    import argparse

    import torch.distributed as dist

    from dstraining_b200.trainer import Trainer, add_args
    from dstraining_b200.utils import checkpoint

    monkeypatch.setenv("DST_INIT_METHOD", f"file://{tmp_path}/store")
    monkeypatch.setenv("RANK", "0")
    monkeypatch.setenv("WORLD_SIZE", "1")
    argv = ["--bf16", "--vp", "--layers", "2", "--heads", "4", "--embd", "256", "--block", "256", "--vocab", "1000",
            "--batch", "4", "--lr", "1e-3", "--seed", "5"]
    try:
        def run(tr, first, n):
            out = []
            for s in range(first, first + n):
                x, y = tr.shard.get_batch(s)
                out.append(tr.step_device(x.to(cuda), y.to(cuda)).item())
            return out

        a = add_args(argparse.ArgumentParser()).parse_args(argv)
        straight = run(Trainer(a), 0, 6)
        tr = Trainer(add_args(argparse.ArgumentParser()).parse_args(argv))
        assert tr.fused_dp
        first = run(tr, 0, 3)
        path = checkpoint.save(str(tmp_path / "ck"), 3, tr.model, tr.opt, tr.tp, tr.pp, tr.dp, tr.config, 5)
        tr2 = Trainer(add_args(argparse.ArgumentParser()).parse_args(argv))
        checkpoint.load(path, tr2.model, tr2.opt, tr2.tp)
        resumed = first + run(tr2, 3, 3)
        assert max(abs(x - y) for x, y in zip(straight, resumed)) < 1e-3, (straight, resumed)
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()
