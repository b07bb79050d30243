"""Local multi-process launcher: ``python -m dstraining_b200.utils.launch N script.py args...``

Spawns N ranks of a script with ``RANK``/``LOCAL_RANK``/``WORLD_SIZE`` and a
FileStore rendezvous (``DST_INIT_METHOD=file://...``), so multi-rank runs need
no sockets or hostname resolution; exits non-zero if any rank fails, and
kills the survivors if one rank fails or the optional ``--timeout`` expires
(a dead rank must not leave its peers waiting forever). The reference ships
the same launcher as a shell script (``scripts/launch_local.sh``).

Automatic restart (``--max-restarts K --restart-args "--resume"``): when the
job fails, every rank is stopped and the whole job is launched again (a new
rendezvous) with the restart arguments appended, up to K times - with
``train.py --ckpt-dir ... --ckpt-every ...`` this resumes from the latest
complete checkpoint, the recovery path after a rank failure. With
``--restart-nproc M`` (and layout flags in ``--restart-args``) the job comes
back on M ranks: checkpoints are resharded on load. SIGTERM / SIGUSR1 to the
launcher go to every rank, and a job stopped that way is not restarted.
"""

from __future__ import annotations

import argparse
import os
import shlex
import signal
import subprocess
import sys
import tempfile
import time
from typing import List, Optional, Sequence


_FORWARDED: List[int] = []  # signals passed on to the ranks (a preempted job is not restarted)


def launch(nproc: int, argv: List[str], timeout: Optional[float] = None, env: Optional[dict] = None) -> int:
    """Run ``nproc`` ranks of ``python argv``; 0 if every rank exits 0, else 1
    (survivors are killed when one fails or the timeout expires). SIGTERM and
    SIGUSR1 sent to the launcher are passed on to every rank (with
    ``train.py --save-on-signal`` they checkpoint together and exit 0)."""
    store_dir = tempfile.mkdtemp(prefix="dst_store_")
    store = os.path.join(store_dir, "store")
    procs = []
    for r in range(nproc):
        e = dict(os.environ if env is None else env)
        e.update(RANK=str(r), LOCAL_RANK=str(r), WORLD_SIZE=str(nproc), DST_INIT_METHOD=f"file://{store}")
        procs.append(subprocess.Popen([sys.executable, *argv], env=e, start_new_session=True))

    def forward(signum, frame):  # noqa: ARG001 - signal handler signature
        _FORWARDED.append(signum)
        for p in procs:
            if p.poll() is None:
                try:
                    os.killpg(p.pid, signum)
                except ProcessLookupError:
                    pass

    previous = {}
    for sig in (signal.SIGTERM, signal.SIGUSR1):
        try:
            previous[sig] = signal.signal(sig, forward)
        except ValueError:  # not the main thread: leave signals alone
            pass
    deadline = None if timeout is None else time.monotonic() + timeout
    codes = [None] * nproc
    try:
        while any(c is None for c in codes):
            for i, p in enumerate(procs):
                if codes[i] is None:
                    codes[i] = p.poll()
            failed = any(c not in (None, 0) for c in codes)
            expired = deadline is not None and time.monotonic() > deadline
            if failed or expired:
                for i, p in enumerate(procs):
                    if codes[i] is None:
                        os.killpg(p.pid, signal.SIGKILL)
                        p.wait()
                        codes[i] = -9
                break
            time.sleep(0.05)
    finally:
        for p in procs:
            if p.poll() is None:
                os.killpg(p.pid, signal.SIGKILL)
        for sig, handler in previous.items():
            signal.signal(sig, handler)
    return 0 if all(c == 0 for c in codes) else 1


def launch_with_restarts(nproc: int, argv: List[str], max_restarts: int = 0, restart_args: Sequence[str] = (),
                         timeout: Optional[float] = None, env: Optional[dict] = None,
                         restart_nproc: Optional[int] = None) -> int:
    """:func:`launch`, relaunching the whole job after a failure (at most
    ``max_restarts`` times) with ``restart_args`` appended (later flags win, so
    they may also change the layout, e.g. ``--resume --tp 1``) and, if given,
    ``restart_nproc`` ranks - an elastic restart on fewer (or more) GPUs from
    the reshardable checkpoint. Returns 0 once an attempt succeeds, 1 when
    every attempt failed."""
    for attempt in range(max_restarts + 1):
        args = list(argv) if attempt == 0 else [*argv, *restart_args]
        n = nproc if attempt == 0 or restart_nproc is None else restart_nproc
        if launch(n, args, timeout, env) == 0:
            return 0
        if _FORWARDED:
            print("[dst launch] stopped by a signal; not restarting", file=sys.stderr, flush=True)
            return 1
        if attempt < max_restarts:
            print(f"[dst launch] job failed; restart {attempt + 1} of {max_restarts}", file=sys.stderr, flush=True)
    return 1


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--timeout", type=float, default=None, help="per attempt")
    ap.add_argument("--max-restarts", type=int, default=0)
    ap.add_argument("--restart-args", default="", help="arguments appended on restarts, e.g. \"--resume\"")
    ap.add_argument("--restart-nproc", type=int, default=None, help="ranks for restarts (elastic; default: nproc)")
    ap.add_argument("nproc", type=int)
    ap.add_argument("argv", nargs=argparse.REMAINDER)
    a = ap.parse_args()
    sys.exit(launch_with_restarts(a.nproc, a.argv, a.max_restarts, shlex.split(a.restart_args), a.timeout,
                                  restart_nproc=a.restart_nproc))


if __name__ == "__main__":
    main()
