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


def test_step_gate_raises_on_missing_rank(one_rank):
    gate = health.StepGate(timeout=0.3)
    t0 = time.time()
    with pytest.raises(health.PeerFailure, match=r"\[1\] did not reach step 0"):
        gate.enter(0)
    assert time.time() - t0 < 5
