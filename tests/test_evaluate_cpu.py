"""Checkpoint evaluation: the loss over consecutive windows equals the
model's own loss on those windows, batching does not change it, and the CLI
reads a checkpoint written at tp=2."""

import json
import math
import os

import numpy as np
import torch

from dstraining_b200.models.gpt import GPT, GPTConfig
from dstraining_b200.parallel.topology import SINGLE
from dstraining_b200.utils.evaluate import evaluate, main
from dstraining_b200.utils.launch import launch


def test_matches_model_loss(tmp_path):
    cfg = GPTConfig(vocab_size=200, block_size=16, n_layer=1, n_head=2, n_embd=32)
    m = GPT(cfg, SINGLE, seed=4)
    data = (np.arange(16 * 5 + 3) * 7 % 200).astype(np.uint16)
    data.tofile(tmp_path / "v.bin")
    out = evaluate(m, str(tmp_path / "v.bin"), batch=2)
    assert out["tokens"] == 5 * 16
    rows = torch.from_numpy(np.stack([data[s : s + 17] for s in range(0, 5 * 16, 16)]).astype(np.int64))
    with torch.no_grad():
        _, want = m(rows[:, :-1], rows[:, 1:])
    assert abs(out["loss"] - float(want)) < 1e-5 and abs(out["perplexity"] - math.exp(out["loss"])) < 1e-6
    assert abs(evaluate(m, str(tmp_path / "v.bin"), batch=5)["loss"] - out["loss"]) < 1e-5
    assert evaluate(m, str(tmp_path / "v.bin"), batch=2, max_tokens=32)["tokens"] == 32


def test_cli_from_tp2_checkpoint(tmp_path, capsys):
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="1")
    argv = [os.path.join(root, "train.py"), "--tp", "2", "--layers", "1", "--heads", "2", "--embd", "32",
            "--block", "32", "--vocab", "128", "--batch", "2", "--steps", "2", "--device", "cpu",
            "--ckpt-dir", str(tmp_path / "ck")]
    assert launch(2, argv, timeout=300, env=env) == 0
    (np.arange(500) % 128).astype(np.uint16).tofile(tmp_path / "v.bin")
    main(["--ckpt", str(tmp_path / "ck"), "--data", str(tmp_path / "v.bin"), "--device", "cpu"])
    out = json.loads(capsys.readouterr().out)
    assert out["tokens"] == 15 * 32 and out["loss"] > 0
