"""Token data: with one file the draws are the reference's single-file draws
(``randint(len - block - 1)`` from the ``seed*1000003 + step*1009 + dp_rank``
generator); several files (directory, glob, list) give windows that lie
inside one file, deterministic per (seed, step, dp rank)."""

import numpy as np
import torch

from dstraining_b200.parallel.topology import TPContext
from dstraining_b200.utils.data import TokenShard


def test_single_file_matches_reference_draw(tmp_path):
    data = np.arange(5000, dtype=np.uint16) % 997
    data.tofile(tmp_path / "a.bin")
    x, y = TokenShard(str(tmp_path / "a.bin"), 32, 4, seed=3).get_batch(7)
    g = torch.Generator().manual_seed(3 * 1000003 + 7 * 1009 + 0)
    starts = torch.randint(5000 - 32 - 1, (4,), generator=g)
    want = torch.stack([torch.from_numpy(data[s : s + 33].astype(np.int64)) for s in starts.tolist()])
    assert torch.equal(x, want[:, :-1]) and torch.equal(y, want[:, 1:])


def test_several_files(tmp_path):
    sizes = {"a.bin": 300, "b.bin": 40, "c.bin": 10}  # c.bin is shorter than a window: never drawn
    for i, (name, n) in enumerate(sizes.items()):
        np.full(n, i, dtype=np.uint16).tofile(tmp_path / name)
    dp = TPContext(group=None, rank=1, world=2)
    for spec in (str(tmp_path), str(tmp_path / "*.bin"), ",".join(str(tmp_path / n) for n in sizes)):
        shard = TokenShard(spec, 16, 64, seed=0, dp=dp)
        assert len(shard.files) == 3 and shard.counts == [283, 23, 0]
        x, y = shard.get_batch(5)
        rows = torch.cat([x, y[:, -1:]], dim=1)
        assert bool((rows == rows[:, :1]).all())  # every window inside one file
        assert set(rows[:, 0].tolist()) == {0, 1}
        x2, _ = TokenShard(spec, 16, 64, seed=0, dp=dp).get_batch(5)
        assert torch.equal(x, x2)
