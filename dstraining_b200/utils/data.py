"""Training data: a memory-mapped token shard, or synthetic tokens.

Both sources are pure functions of ``(seed, step, dp_rank)``: the generator
for step ``k`` on data-parallel replica ``d`` is seeded
``seed * 1000003 + k * 1009 + d`` (the reference's contract,
``dst/data.py:35-37,61-63``). Every TP rank and pipeline stage of one replica
therefore draws the identical batch with no broadcast, replicas draw
different batches, and resuming at step ``k`` needs no saved loader state.

``TokenShard`` reads a flat uint16 token file (nanoGPT format) through
``np.memmap``; targets are the inputs shifted by one. ``SyntheticShard``
draws inputs and targets as independent uniform ids.

``get_batch(step, pin=True)`` returns CPU tensors in pinned memory, so the
host->device copy that starts a training step can be asynchronous.
"""

from __future__ import annotations

import numpy as np
import torch

from ..parallel.topology import DP_SINGLE, DPContext


def _generator(seed: int, step: int, dp: DPContext) -> torch.Generator:
    return torch.Generator().manual_seed(seed * 1000003 + step * 1009 + dp.rank)


def _maybe_pin(t: torch.Tensor, pin: bool) -> torch.Tensor:
    return t.pin_memory() if pin and torch.cuda.is_available() else t


class TokenShard:
    """Random windows of a flat uint16 token file (``dst/data.py:23-45``); targets
    are inputs shifted by one; batches are a pure function of (seed, step, dp rank)."""

    def __init__(self, path: str, block_size: int, batch_size: int, seed: int = 0, dp: DPContext = DP_SINGLE):
        self.data = np.memmap(path, dtype=np.uint16, mode="r")
        if len(self.data) < block_size + 1:
            raise ValueError(f"shard {path} shorter than one block")
        self.block_size, self.batch_size, self.seed, self.dp = block_size, batch_size, seed, dp

    def get_batch(self, step: int, pin: bool = False):
        g = _generator(self.seed, step, self.dp)
        starts = torch.randint(len(self.data) - self.block_size - 1, (self.batch_size,), generator=g)
        rows = np.stack([np.asarray(self.data[s : s + self.block_size + 1]) for s in starts.tolist()])
        rows = torch.from_numpy(rows.astype(np.int64))
        return _maybe_pin(rows[:, :-1].contiguous(), pin), _maybe_pin(rows[:, 1:].contiguous(), pin)


class SyntheticShard:
    """Uniform-random token ids and targets (``dst/data.py:48-66``), seeded like TokenShard."""

    def __init__(self, vocab_size: int, block_size: int, batch_size: int, seed: int = 0, dp: DPContext = DP_SINGLE):
        self.vocab_size, self.block_size, self.batch_size, self.seed, self.dp = (
            vocab_size,
            block_size,
            batch_size,
            seed,
            dp,
        )

    def get_batch(self, step: int, pin: bool = False):
        g = _generator(self.seed, step, self.dp)
        shape = (self.batch_size, self.block_size)
        x = torch.randint(self.vocab_size, shape, generator=g)
        y = torch.randint(self.vocab_size, shape, generator=g)
        return _maybe_pin(x, pin), _maybe_pin(y, pin)
