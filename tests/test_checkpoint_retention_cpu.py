"""Checkpoint retention (``--ckpt-keep``): only the newest N complete
checkpoints stay; failed (incomplete) writes older than the newest complete
checkpoint go too, newer incomplete ones (a background write in progress)
stay."""

import os

from dstraining_b200.utils import checkpoint
from dstraining_b200.utils.launch import launch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _mk(root, step, complete):
    d = root / f"step_{step:08d}"
    d.mkdir()
    (d / "shard_tp0_pp0.pt").write_bytes(b"x")
    if complete:
        (d / "COMPLETE").write_text("ok\n")


def test_prune(tmp_path):
    for step, complete in ((2, True), (4, False), (6, True), (8, True), (10, True), (12, False)):
        _mk(tmp_path, step, complete)
    (tmp_path / "notes.txt").write_text("kept")
    removed = checkpoint.prune(str(tmp_path), 2)
    assert sorted(os.path.basename(p) for p in removed) == ["step_00000002", "step_00000004", "step_00000006"]
    assert sorted(os.listdir(tmp_path)) == ["notes.txt", "step_00000008", "step_00000010", "step_00000012"]
    assert checkpoint.latest(str(tmp_path)).endswith("step_00000010")
    assert checkpoint.prune(str(tmp_path), 0) == []  # 0: keep everything


def test_train_keeps_newest(tmp_path):
    ck = tmp_path / "ck"
    args = [os.path.join(ROOT, "train.py"), "--device", "cpu", "--layers", "1", "--heads", "2", "--embd", "32",
            "--block", "16", "--vocab", "128", "--batch", "2", "--steps", "5", "--ckpt-dir", str(ck),
            "--ckpt-every", "1", "--ckpt-keep", "2", "--log-every", "5"]
    env = dict(os.environ, PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""))
    assert launch(1, [*args, "--ckpt-async"], timeout=240, env=env) == 0
    assert sorted(os.listdir(ck)) == ["step_00000004", "step_00000005"]
