"""Health primitives in one process: a one-rank gloo group whose world size
is reported as 2, so "rank 1" never publishes - the watchdog must name it,
the step gate must raise, and a failure record must be seen."""

import time

import pytest
import torch.distributed as dist

from dstraining_b200.parallel import health


@pytest.fixture
def one_rank(tmp_path, monkeypatch):
    dist.init_process_group("gloo", init_method=f"file://{tmp_path}/store", rank=0, world_size=1)
    monkeypatch.setattr(health.dist, "get_world_size", lambda *a, **k: 2)
    yield
    dist.destroy_process_group()


def test_watchdog_names_silent_peer(one_rank):
    hb = health.Heartbeat(interval=0.05).start()
    seen = []
    wd = health.Watchdog(timeout=0.3, poll=0.05, grace=0.1, on_failure=seen.append).start()
    t0 = time.time()
    while not seen and time.time() - t0 < 5:
        time.sleep(0.05)
    hb.stop()
    wd.stop()
    assert seen == [[1]] and wd.failed == [1]


def test_stale_and_failed_ranks(one_rank):
    hb = health.Heartbeat(interval=10.0)  # publishes once at construction
    assert health.stale_ranks(5.0) == [1]  # rank 1 never published
    hb.last -= 100.0
    hb.beat()
    assert health.stale_ranks(5.0) == [0, 1]  # rank 0's last progress is old
    hb.tick()
    hb.beat()
    health.report_failure("boom")
    assert health.stale_ranks(5.0) == [0, 1]  # rank 0 reported a failure


def test_hold_keeps_a_busy_rank_fresh(one_rank):
    """A rank inside a long non-step phase (checkpoint, evaluation) publishes
    the current time, not its last step; its last step counts again after."""
    hb = health.Heartbeat(interval=10.0)
    hb.last -= 100.0
    with hb.hold():
        hb.beat()
        assert 0 not in health.stale_ranks(5.0)
    hb.last -= 100.0  # the phase has ended: no further steps
    hb.beat()
    assert 0 in health.stale_ranks(5.0)


def test_step_gate_raises_on_missing_rank(one_rank):
    gate = health.StepGate(timeout=0.3)
    t0 = time.time()
    with pytest.raises(health.PeerFailure, match=r"\[1\] did not reach step 0"):
        gate.enter(0)
    assert time.time() - t0 < 5


def test_save_on_signal_then_resume(tmp_path):
    """--save-on-signal: rank 1 receives SIGTERM during step 3; at the next
    agreed check (after step 3) every rank checkpoints step 4 and exits 0;
    --resume continues from it to the end."""
    import os

    from dstraining_b200.utils import checkpoint
    from dstraining_b200.utils.launch import launch

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    ck = str(tmp_path / "ck")
    common = [os.path.join(root, "train.py"), "--dp", "2", "--layers", "1", "--heads", "2", "--embd", "32",
              "--block", "32", "--vocab", "128", "--batch", "2", "--steps", "12", "--device", "cpu",
              "--ckpt-dir", ck, "--save-on-signal", "--signal-check-every", "2"]
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="1", DST_INJECT_SIGNAL="1:3")
    assert launch(2, common, timeout=300, env=env) == 0
    assert checkpoint.latest(ck).endswith("step_00000004")
    env.pop("DST_INJECT_SIGNAL")
    assert launch(2, [*common, "--resume"], timeout=300, env=env) == 0
    assert checkpoint.latest(ck).endswith("step_00000012")


def test_time_limit_checkpoints_and_exits(tmp_path):
    import os

    from dstraining_b200.utils import checkpoint
    from dstraining_b200.utils.launch import launch

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    ck = str(tmp_path / "ck")
    argv = [os.path.join(root, "train.py"), "--layers", "1", "--heads", "2", "--embd", "32", "--block", "32",
            "--vocab", "128", "--batch", "2", "--steps", "100000", "--device", "cpu", "--ckpt-dir", ck,
            "--time-limit-min", "0.0001", "--signal-check-every", "3"]
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="1")
    assert launch(1, argv, timeout=300, env=env) == 0
    assert checkpoint.latest(ck).endswith("step_00000003")  # the first check, past 6 ms


def test_launcher_forwards_sigterm(tmp_path):
    """SIGTERM to the launcher reaches every rank; with --save-on-signal the
    job checkpoints at an agreed step and the launcher exits 0."""
    import os
    import signal
    import subprocess
    import sys
    import time

    from dstraining_b200.utils import checkpoint

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    ck = str(tmp_path / "ck")
    sink = tmp_path / "m.jsonl"
    cmd = [sys.executable, "-m", "dstraining_b200.utils.launch", "--timeout", "240", "2",
           os.path.join(root, "train.py"), "--dp", "2", "--layers", "1", "--heads", "2", "--embd", "32", "--block",
           "32", "--vocab", "128", "--batch", "2", "--steps", "100000", "--device", "cpu", "--ckpt-dir", ck,
           "--save-on-signal", "--signal-check-every", "2", "--jsonl", str(sink)]
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="1",
               PYTHONPATH=root + os.pathsep + os.environ.get("PYTHONPATH", ""))
    p = subprocess.Popen(cmd, env=env, cwd=root)
    try:
        t0 = time.time()
        while not (sink.exists() and len(sink.read_text().splitlines()) >= 3):
            assert p.poll() is None and time.time() - t0 < 120
            time.sleep(0.2)
        p.send_signal(signal.SIGTERM)
        assert p.wait(timeout=120) == 0
    finally:
        if p.poll() is None:
            p.kill()
    assert checkpoint.latest(ck) is not None
