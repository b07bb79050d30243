"""Training data: a memory-mapped token shard, or synthetic tokens.

Both sources are pure functions of ``(seed, step, dp_rank)``: the generator
for step ``k`` on data-parallel replica ``d`` is seeded
``seed * 1000003 + k * 1009 + d`` (the reference's contract,
``dst/data.py:35-37,61-63``). Every TP rank and pipeline stage of one replica
therefore draws the identical batch with no broadcast, replicas draw
different batches, and resuming at step ``k`` needs no saved loader state.

``TokenShard`` reads a flat uint16 token file (nanoGPT format) through
``np.memmap``; targets are the inputs shifted by one. It also takes several
files (a directory of ``.bin`` files, a glob pattern or a comma-separated
list): windows are then drawn uniformly over all files' window positions
and never cross a file boundary; with one file the draws are exactly the
single-file ones. ``SyntheticShard`` draws inputs and targets as
independent uniform ids.

``get_batch(step, pin=True)`` returns CPU tensors in pinned memory, so the
host->device copy that starts a training step can be asynchronous.
"""

from __future__ import annotations

import glob
import os
from typing import List

import numpy as np
import torch

from ..parallel.topology import DP_SINGLE, DPContext


def _generator(seed: int, step: int, dp: DPContext) -> torch.Generator:
    return torch.Generator().manual_seed(seed * 1000003 + step * 1009 + dp.rank)


def _maybe_pin(t: torch.Tensor, pin: bool) -> torch.Tensor:
    return t.pin_memory() if pin and torch.cuda.is_available() else t


def token_files(path: str) -> List[str]:
    """The token files named by ``path``: a file, a directory (its ``.bin``
    files), a glob pattern or a comma-separated list of those; sorted."""
    out: List[str] = []
    for part in path.split(","):
        if os.path.isdir(part):
            out += sorted(os.path.join(part, f) for f in os.listdir(part) if f.endswith(".bin"))
        elif any(c in part for c in "*?["):
            out += sorted(glob.glob(part))
        else:
            out.append(part)
    if not out:
        raise ValueError(f"no token files in {path!r}")
    return out


class TokenShard:
    """Random windows of flat uint16 token files (``dst/data.py:23-45``); targets
    are inputs shifted by one; batches are a pure function of (seed, step, dp rank)."""

    def __init__(self, path: str, block_size: int, batch_size: int, seed: int = 0, dp: DPContext = DP_SINGLE):
        self.files = token_files(path)
        self.maps = [np.memmap(f, dtype=np.uint16, mode="r") for f in self.files]
        # window starts per file: [0, len - block - 1), as in the single-file draw
        self.counts = [max(0, len(m) - block_size - 1) for m in self.maps]
        if not any(self.counts):
            raise ValueError(f"{path}: no file longer than one block")
        self.offsets = np.cumsum([0] + self.counts)
        self.data = self.maps[0]  # the single-file attribute of earlier versions
        self.block_size, self.batch_size, self.seed, self.dp = block_size, batch_size, seed, dp

    def get_batch(self, step: int, pin: bool = False):
        g = _generator(self.seed, step, self.dp)
        starts = torch.randint(int(self.offsets[-1]), (self.batch_size,), generator=g)
        rows = []
        for s in starts.tolist():
            f = int(np.searchsorted(self.offsets, s, side="right")) - 1
            o = s - int(self.offsets[f])
            rows.append(np.asarray(self.maps[f][o : o + self.block_size + 1]))
        rows = torch.from_numpy(np.stack(rows).astype(np.int64))
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
