"""A rank leaves between steps; the others notice on the host, before their
next step launches anything (``Trainer`` with ``--step-gate-timeout``).

    python -m dstraining_b200.utils.launch 2 tests/suites/gate_suite.py --marker /tmp/m
    torchrun --nproc-per-node 2 tests/suites/gate_suite.py --device cuda --marker /tmp/m

The victim finishes step 3 completely (on CUDA: its device synchronised, so
every fused-collective kernel that involves it has finished on all ranks),
then exits with status 0 without entering step 4. Survivors block in the
step gate of step 4, get ``PeerFailure`` after the gate timeout, leave a
marker file and exit with status 3: no kernel or collective of step 4 was
ever launched, so nothing on the device waits for the departed rank.
"""

import argparse
import os
import sys
import time

import common  # noqa: F401  (puts the repository on sys.path)
import dstraining_b200  # noqa: F401  (sets kernel loading before CUDA starts)
import torch
import torch.distributed as dist

from dstraining_b200.parallel.health import PeerFailure
from dstraining_b200.trainer import Trainer, add_args


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--device", default="cpu")
    ap.add_argument("--victim", type=int, default=1)
    ap.add_argument("--marker", default=None)
    ap.add_argument("--gate-timeout", type=float, default=5.0)
    a = ap.parse_args()
    os.environ.setdefault("DST_PG_TIMEOUT_S", "120")  # the gate must fire first
    cuda = a.device == "cuda"
    argv = ["--dp", os.environ.get("WORLD_SIZE", "2"), "--layers", "1", "--heads", "2", "--embd", "128",
            "--block", "128", "--vocab", "512", "--batch", "4", "--device", a.device,
            "--step-gate-timeout", str(a.gate_timeout)]
    if cuda:
        argv += ["--bf16", "--vp"]  # native kernels and the fused NVLink DP optimizer
    tr = Trainer(add_args(argparse.ArgumentParser()).parse_args(argv))
    rank = dist.get_rank()
    for step in range(8):
        if rank == a.victim and step == 4:
            if cuda:
                torch.cuda.synchronize()
            print(f"rank {rank}: leaving after step 3", flush=True)
            os._exit(0)
        x, y = tr.shard.get_batch(step)
        try:
            t0 = time.time()
            tr.step_device(x.to(tr.device), y.to(tr.device))
        except PeerFailure as e:
            waited = time.time() - t0
            print(f"rank {rank}: {e} (noticed after {waited:.1f} s, before launching step {step})", flush=True)
            if a.marker:
                with open(f"{a.marker}.{rank}", "w") as f:
                    f.write(f"{step} {e}\n")
            os._exit(3)
        if cuda:
            torch.cuda.synchronize()
    print(f"rank {rank}: no failure observed", flush=True)
    sys.exit(1)


if __name__ == "__main__":
    main()
