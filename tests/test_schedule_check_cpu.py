"""Deadlock freedom of the pipeline schedules for every (stages, chunks,
micro-batches) up to 8 x 4 x 16, played from the op orders the schedules
execute; the checker itself catches a schedule that does deadlock."""

import pytest

from dstraining_b200.parallel.pipeline import order_1f1b, order_interleaved
from dstraining_b200.parallel.schedule_check import check, main, simulate


def _cases():
    for p in range(1, 9):
        for v in range(1, 5):
            for m in range(1, 17):
                if v == 1 or m % p == 0:
                    yield p, v, m


def test_all_schedules_complete():
    bad = [(p, v, m) for p, v, m in _cases() if not check(p, v, m)["ok"]]
    assert not bad


def test_orders_cover_every_step_once():
    for p, v, m in _cases():
        for r in range(p):
            ops = order_interleaved(p, r, v, m) if v > 1 else order_1f1b(p, r, m)
            n = m * v
            assert sorted(k for op, k in ops if op == "F") == list(range(n))
            assert sorted(k for op, k in ops if op == "B") == list(range(n))
            # a backward never comes before its forward
            seen = set()
            for op, k in ops:
                if op == "F":
                    seen.add(k)
                else:
                    assert k in seen


def test_checker_detects_deadlock():
    # both ranks wait for the other first: no delivery model completes this
    progs = [[("recv", ("fwd", 1, 0)), ("send", ("fwd", 0, 1))], [("recv", ("fwd", 0, 1)), ("send", ("fwd", 1, 0))]]
    out = simulate(progs)
    assert not out["ok"] and set(out["stuck"]) == {0, 1}
    # 1F1B needs sends that do not wait for their receiver: without buffering its
    # steady state (a forward send against a backward send) stops
    assert check(2, 1, 2)["ok"] and not check(2, 1, 2, "rendezvous")["ok"]
    # a message nobody receives is reported
    assert simulate([[("send", ("fwd", 0, 1))], []])["undelivered"]


def test_cli():
    with pytest.raises(SystemExit) as e:
        main(["--pp", "4", "--chunks", "2", "--micro-batches", "8"])
    assert e.value.code == 0
