"""Trainer / train.py plumbing on CPU (fp32 oracle path)."""

import argparse
import os

import pytest
import torch


@pytest.fixture()
def single_rank(monkeypatch, tmp_path):
    import torch.distributed as dist

    monkeypatch.setenv("DST_INIT_METHOD", f"file://{tmp_path}/store")
    monkeypatch.setenv("RANK", "0")
    monkeypatch.setenv("WORLD_SIZE", "1")
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "")
    yield
    if dist.is_initialized():
        dist.destroy_process_group()


def test_trainer_loss_falls(single_rank):
    from dstraining_b200.trainer import Trainer, add_args

    a = add_args(argparse.ArgumentParser()).parse_args(["--device", "cpu", "--layers", "2", "--batch", "4", "--lr", "1e-3"])
    tr = Trainer(a)
    x, y = tr.shard.get_batch(0)
    losses = [tr.step(x, y) for _ in range(8)]
    assert losses[-1] < losses[0]
    assert tr.tokens_per_step == 4 * 64
