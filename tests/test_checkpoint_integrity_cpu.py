"""Checkpoint integrity: every shard carries a SHA-256, ``inspect`` reports a
checkpoint as whole, and a corrupted shard is refused on load."""

import json

import pytest
import torch

from dstraining_b200.models.gpt import GPT, GPTConfig
from dstraining_b200.parallel.topology import PP_SINGLE, SINGLE
from dstraining_b200.utils import checkpoint


def _model():
    return GPT(GPTConfig(vocab_size=256, block_size=16, n_layer=1, n_head=2, n_embd=32), SINGLE, seed=3)


def test_checksums_inspect_and_corruption(tmp_path, capsys):
    m = _model()
    opt = torch.optim.Adam(m.parameters(), lr=1e-3)
    path = checkpoint.save(str(tmp_path), 7, m, opt, SINGLE, PP_SINGLE, SINGLE, m.config, 3)
    info = checkpoint.inspect(path)
    assert info["ok"] and info["step"] == 7 and info["tensors"] > 0 and not info["corrupt"]
    with pytest.raises(SystemExit) as e:
        checkpoint.main([str(tmp_path)])  # a root resolves to its latest checkpoint
    assert e.value.code == 0 and json.loads(capsys.readouterr().out)["ok"]

    m2 = _model()
    checkpoint.load(path, m2, None, SINGLE)  # intact: loads
    shard = tmp_path / "step_00000007" / "shard_tp0_pp0.pt"
    raw = bytearray(shard.read_bytes())
    raw[len(raw) // 2] ^= 0xFF
    shard.write_bytes(bytes(raw))
    assert checkpoint.inspect(path)["corrupt"] == ["shard_tp0_pp0.pt"]
    with pytest.raises(RuntimeError, match="SHA-256"):
        checkpoint.load(path, _model(), None, SINGLE)


def test_background_write_error_surfaces(tmp_path, monkeypatch):
    """A failing background write is re-raised by wait() and leaves no
    COMPLETE marker, so ``latest`` never picks the broken checkpoint."""
    m = _model()

    def broken_save(*a, **k):
        raise OSError("disk full")

    monkeypatch.setattr(checkpoint.torch, "save", broken_save)
    pending = checkpoint.save(str(tmp_path), 9, m, None, SINGLE, PP_SINGLE, SINGLE, m.config, 3, background=True)
    with pytest.raises(RuntimeError, match="failed") as e:
        pending.wait()
    assert isinstance(e.value.__cause__, OSError)
    assert checkpoint.latest(str(tmp_path)) is None
