"""Learning-rate schedule: warm-up then cosine, applied by the trainer before
each step, to every optimizer kind."""

import argparse
import math

import torch

from dstraining_b200.optim.schedule import lr_at, set_lr


def test_lr_at():
    assert [lr_at(s, 1.0, 10, warmup_steps=4) for s in range(4)] == [0.25, 0.5, 0.75, 1.0]
    assert lr_at(4, 1.0, 10, 4, "cosine", 0.1) == 1.0
    assert math.isclose(lr_at(7, 1.0, 10, 4, "cosine", 0.1), 0.1 + 0.45 * (1 + math.cos(math.pi * 0.5)))
    assert math.isclose(lr_at(10, 1.0, 10, 4, "cosine", 0.1), 0.1)
    assert lr_at(50, 1.0, 10, 0, "constant") == 1.0


def test_set_lr_on_optimizers():
    from dstraining_b200.optim.precision import MasterWeightOptimizer

    p = torch.nn.Parameter(torch.zeros(4))
    adam = torch.optim.Adam([p], lr=1.0)
    set_lr(adam, 0.5)
    assert adam.param_groups[0]["lr"] == 0.5
    mw = MasterWeightOptimizer([torch.nn.Parameter(torch.zeros(4))], lr=1.0)
    set_lr(mw, 0.25)
    assert mw.inner.param_groups[0]["lr"] == 0.25

    class Fused:
        lr = 1.0

    f = Fused()
    set_lr(f, 0.125)
    assert f.lr == 0.125


def test_trainer_applies_schedule(monkeypatch, tmp_path):
    import torch.distributed as dist

    from dstraining_b200.trainer import Trainer, add_args

    monkeypatch.setenv("DST_INIT_METHOD", f"file://{tmp_path}/store")
    monkeypatch.setenv("RANK", "0")
    monkeypatch.setenv("WORLD_SIZE", "1")
    argv = ["--layers", "1", "--heads", "2", "--embd", "32", "--block", "16", "--vocab", "64", "--batch", "2",
            "--device", "cpu", "--steps", "6", "--lr", "1e-3", "--warmup-steps", "2", "--lr-schedule", "cosine"]
    try:
        tr = Trainer(add_args(argparse.ArgumentParser()).parse_args(argv))
        seen = []
        for s in range(6):
            x, y = tr.shard.get_batch(s)
            tr.step_device(x, y)
            seen.append(tr.opt.param_groups[0]["lr"])
        want = [lr_at(s, 1e-3, 6, 2, "cosine") for s in range(6)]
        assert all(math.isclose(a, b) for a, b in zip(seen, want)), (seen, want)
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()
