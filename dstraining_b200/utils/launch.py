"""Local multi-process launcher: ``python -m dstraining_b200.utils.launch N script.py args...``

Spawns N ranks of a script with ``RANK``/``LOCAL_RANK``/``WORLD_SIZE`` and a
FileStore rendezvous (``DST_INIT_METHOD=file://...``), so multi-rank runs need
no sockets or hostname resolution; exits non-zero if any rank fails, and
kills the survivors if one rank fails or the optional ``--timeout`` expires
(a dead rank must not leave its peers waiting forever). The reference ships
the same launcher as a shell script (``scripts/launch_local.sh``).
"""

from __future__ import annotations

import argparse
import os
import signal
import subprocess
import sys
import tempfile
import time
from typing import List, Optional


def launch(nproc: int, argv: List[str], timeout: Optional[float] = None, env: Optional[dict] = None) -> int:
    store_dir = tempfile.mkdtemp(prefix="dst_store_")
    store = os.path.join(store_dir, "store")
    procs = []
    for r in range(nproc):
        e = dict(os.environ if env is None else env)
        e.update(RANK=str(r), LOCAL_RANK=str(r), WORLD_SIZE=str(nproc), DST_INIT_METHOD=f"file://{store}")
        procs.append(subprocess.Popen([sys.executable, *argv], env=e, start_new_session=True))
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
    return 0 if all(c == 0 for c in codes) else 1


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--timeout", type=float, default=None)
    ap.add_argument("nproc", type=int)
    ap.add_argument("argv", nargs=argparse.REMAINDER)
    a = ap.parse_args()
    sys.exit(launch(a.nproc, a.argv, a.timeout))


if __name__ == "__main__":
    main()
