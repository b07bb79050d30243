"""Failure detection for multi-rank training (host side).

Three layers, none of which needs a GPU fault to be exercised:

* a short, configurable process-group timeout (``DST_PG_TIMEOUT_S``, set in
  :func:`dstraining_b200.parallel.topology.init_distributed`): a collective
  whose peer died or stalled ends with an error instead of waiting forever;
* :class:`Heartbeat`: every rank publishes a timestamp into the rendezvous
  store (the c10d store every rank already shares) every ``interval`` seconds
  from a daemon thread;
* :class:`Watchdog`: a daemon thread that reads every rank's heartbeat and,
  when one is older than ``timeout`` (or a rank has posted a failure
  record), reports it and by default terminates this process with exit code
  3 - so a survivor does not sit in a collective until the much longer
  process-group timeout, and the launcher sees the job fail.

``report_failure(reason)`` lets a rank that catches an exception tell its
peers before it exits. :class:`StepGate` checks, on the host and before a
step launches anything, that every rank has reached that step. Device-side waits are bounded inside the kernels
(status word, see ``read_status``); this module covers ranks.

The reference has no failure handling (its only guard is
``GradReducer.finish`` launching never-launched buckets, ``dst/dp.py:134-138``).
"""

from __future__ import annotations

import contextlib
import datetime
import os
import signal
import sys
import threading
import time
from typing import Callable, List, Optional

import torch
import torch.distributed as dist

_PREFIX = "dst/health"


def _store():
    return dist.distributed_c10d._get_default_store()


class PeerFailure(RuntimeError):
    """A peer rank stopped making progress, reported a failure, or missed a step gate."""

    pass


class Heartbeat:
    """Publishes this rank's last *progress* time. The training loop calls
    :meth:`tick` once per step; a daemon thread writes the latest tick into
    the store every ``interval`` seconds (so a slow store never stalls the
    step). A rank whose main loop hangs stops ticking; a rank that dies stops
    publishing; either way its entry goes stale."""

    def __init__(self, interval: float = 1.0):
        self.interval = interval
        self.rank = dist.get_rank()
        self.last = time.time()
        self._held = 0
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, name="dst-heartbeat", daemon=True)
        self.beat()

    def tick(self) -> None:
        self.last = time.time()

    @contextlib.contextmanager
    def hold(self):
        """A long phase that is not a training step (a checkpoint write, an
        evaluation): while it runs the published time keeps moving, so peers
        do not take the rank for hung; progress is ticked when it ends."""
        self._held += 1
        try:
            yield
        finally:
            self._held -= 1
            self.tick()

    def beat(self) -> None:
        _store().set(f"{_PREFIX}/hb/{self.rank}", repr(time.time() if self._held else self.last))

    def _run(self) -> None:
        while not self._stop.wait(self.interval):
            try:
                self.beat()
            except Exception:  # noqa: BLE001 - store gone: the job is ending
                return

    def start(self) -> "Heartbeat":
        self._thread.start()
        return self

    def stop(self) -> None:
        self._stop.set()


def report_failure(reason: str) -> None:
    """Tell every rank that this rank has failed (best effort)."""
    try:
        _store().set(f"{_PREFIX}/failed/{dist.get_rank()}", reason[:200])
        _store().add(f"{_PREFIX}/nfailed", 1)
    except Exception:  # noqa: BLE001
        pass


def stale_ranks(timeout: float, world: Optional[int] = None) -> List[int]:
    """Ranks whose last heartbeat is older than ``timeout`` seconds (or that
    never published one), plus ranks that reported a failure."""
    store = _store()
    world = dist.get_world_size() if world is None else world
    now = time.time()
    bad = []
    failed = int(store.add(f"{_PREFIX}/nfailed", 0))
    for r in range(world):
        if failed:
            try:
                if store.check([f"{_PREFIX}/failed/{r}"]):
                    bad.append(r)
                    continue
            except Exception:  # noqa: BLE001
                pass
        key = f"{_PREFIX}/hb/{r}"
        try:
            if not store.check([key]):
                bad.append(r)
                continue
            t = float(store.get(key).decode())
        except Exception:  # noqa: BLE001
            bad.append(r)
            continue
        if now - t > timeout:
            bad.append(r)
    return bad


class Watchdog:
    """Polls peers' heartbeats; on a stale or failed peer calls ``on_failure``
    (default: print and ``os._exit(3)``)."""

    def __init__(self, timeout: float = 10.0, poll: float = 0.5, on_failure: Optional[Callable[[List[int]], None]] = None,
                 grace: float = 5.0):
        self.timeout = timeout
        self.poll = poll
        self.grace = grace
        self.on_failure = on_failure or self._abort
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, name="dst-watchdog", daemon=True)
        self.failed: List[int] = []

    @staticmethod
    def _abort(ranks: List[int]) -> None:
        print(f"[dst watchdog] rank {dist.get_rank()}: peer rank(s) {ranks} stopped responding; aborting",
              file=sys.stderr, flush=True)
        os._exit(3)

    def _run(self) -> None:
        start = time.time()
        while not self._stop.wait(self.poll):
            if time.time() - start < self.grace:
                continue  # let every rank publish its first heartbeat
            try:
                bad = stale_ranks(self.timeout)
            except Exception:  # noqa: BLE001 - store unreachable: rank 0 (the store host) died
                bad = [0]
            bad = [r for r in bad if r != dist.get_rank()]
            if bad:
                self.failed = bad
                self.on_failure(bad)
                return

    def start(self) -> "Watchdog":
        self._thread.start()
        return self

    def stop(self) -> None:
        self._stop.set()


class StepGate:
    """Host-side rendezvous at the start of every step, before any kernel or
    collective of that step is launched: each rank posts ``step`` to the store
    and waits (at most ``timeout`` seconds) until every rank has posted it.
    A rank that left between steps (exited, crashed, hung on the host) is
    therefore noticed by the others while none of their kernels or
    collectives is in flight, and :meth:`enter` raises :class:`PeerFailure`
    naming the missing ranks. Costs one store round trip per step."""

    def __init__(self, timeout: float = 30.0, prefix: str = f"{_PREFIX}/gate"):
        self.timeout = timeout
        self.prefix = prefix
        self.rank = dist.get_rank()
        self.world = dist.get_world_size()

    def _key(self, step: int, rank: int) -> str:
        return f"{self.prefix}/{step}/{rank}"

    def enter(self, step: int) -> None:
        store = _store()
        store.set(self._key(step, self.rank), "1")
        keys = [self._key(step, r) for r in range(self.world)]
        try:
            store.wait(keys, datetime.timedelta(seconds=self.timeout))
        except Exception as e:  # noqa: BLE001 - store timeout: name the missing ranks
            missing = [r for r in range(self.world) if not store.check([keys[r]])]
            raise PeerFailure(f"rank(s) {missing} did not reach step {step} within {self.timeout:.0f} s") from e
        if step >= 2:  # every rank has passed step - 1, so nobody waits on step - 2 any more
            try:
                store.delete_key(self._key(step - 2, self.rank))
            except Exception:  # noqa: BLE001 - stores without delete keep the key
                pass


def maybe_inject_fault(step: int) -> None:
    """Host-side fault injection for recovery tests: with
    ``DST_INJECT_FAULT="<rank>:<step>"`` that rank raises at the start of that
    step. With ``DST_INJECT_FAULT_ONCE=<file>`` it does so only if the file
    does not exist yet (and creates it), so a restarted job runs through."""
    spec = os.environ.get("DST_INJECT_FAULT")
    if not spec:
        return
    rank, at = (int(v) for v in spec.split(":"))
    if dist.get_rank() != rank or step != at:
        return
    once = os.environ.get("DST_INJECT_FAULT_ONCE")
    if once:
        if os.path.exists(once):
            return
        with open(once, "w") as f:
            f.write(f"rank {rank} step {step}\n")
    raise RuntimeError(f"injected fault on rank {rank} at step {step}")


class StopRequest:
    """Preemption handling: SIGTERM / SIGUSR1 set a flag; :meth:`agreed`
    (a collective over all ranks) tells every rank, at the same step, that at
    least one of them was signalled, so they can checkpoint together and
    exit. ``DST_INJECT_SIGNAL="<rank>:<step>"`` makes that rank signal itself
    at that step (for tests)."""

    def __init__(self, signals=(signal.SIGTERM, signal.SIGUSR1)):
        self.flag = False
        for sig in signals:
            signal.signal(sig, self._handler)

    def _handler(self, signum, frame) -> None:  # noqa: ARG002 - signal handler signature
        self.flag = True

    def maybe_inject(self, step: int) -> None:
        spec = os.environ.get("DST_INJECT_SIGNAL")
        if spec:
            rank, at = (int(v) for v in spec.split(":"))
            if step == at and (not dist.is_initialized() or dist.get_rank() == rank):
                os.kill(os.getpid(), signal.SIGTERM)

    def agreed(self, device: torch.device) -> bool:
        """Whether any rank was signalled (collective: every rank calls it at the same step)."""
        t = torch.tensor([1.0 if self.flag else 0.0], device=device)
        if dist.is_initialized() and dist.get_world_size() > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return bool(t.item() > 0)


def start_monitoring(interval: float = 1.0, timeout: float = 10.0):
    """Heartbeat + watchdog for this rank; returns both (call ``stop()``)."""
    hb = Heartbeat(interval).start()
    wd = Watchdog(timeout=timeout, poll=min(0.5, interval)).start()
    return hb, wd
