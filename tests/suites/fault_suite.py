"""Failure detection on CPU ranks (no GPU is faulted, hung or trapped).

    python -m dstraining_b200.utils.launch 3 tests/suites/fault_suite.py --mode hang --victim 1

Every rank trains a tiny data-parallel model (gloo) with heartbeats and a
watchdog. At step 3 the victim rank fails on the host:

  raise  - the step raises; the rank reports the failure to its peers, exits 1
  hang   - the main loop sleeps forever (no further progress ticks)
  exit   - the process exits with status 0 in the middle of training

Survivors are blocked in their next collective; the watchdog notices the
stale or failed peer and exits them with status 3 well before the
process-group timeout. The launcher therefore returns non-zero quickly.
Rank 0 keeps a marker file so the test can check who detected what.
"""

import argparse
import os
import sys
import time

from common import small_config

import torch
import torch.distributed as dist

from dstraining_b200.models.gpt import GPT
from dstraining_b200.parallel import health, topology
from dstraining_b200.parallel.dp import allreduce_gradients


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--mode", choices=["raise", "hang", "exit"], required=True)
    ap.add_argument("--victim", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--marker", default=None)
    a = ap.parse_args()
    os.environ.setdefault("DST_PG_TIMEOUT_S", "300")  # the watchdog must win, not the PG timeout
    topology.init_distributed(backend="gloo")
    rank = dist.get_rank()
    tp, pp, dp = topology.make_topology(1, 1, dist.get_world_size())
    marker = a.marker

    def on_failure(ranks):
        if marker:
            with open(f"{marker}.{rank}", "w") as f:
                f.write(f"detected {ranks}\n")
        print(f"rank {rank}: detected failed peer(s) {ranks}", flush=True)
        os._exit(3)

    hb = health.Heartbeat(interval=0.2).start()
    wd = health.Watchdog(timeout=2.0, poll=0.2, grace=1.0, on_failure=on_failure).start()
    model = GPT(small_config(n_layer=1), topology.SINGLE, seed=0)
    opt = torch.optim.Adam(model.parameters(), lr=1e-3)
    g = torch.Generator().manual_seed(rank)
    for step in range(a.steps):
        if rank == a.victim and step == 3:
            if a.mode == "raise":
                try:
                    raise RuntimeError("injected failure")
                except RuntimeError as e:
                    health.report_failure(str(e))
                    print(f"rank {rank}: failing on purpose ({e})", flush=True)
                    sys.exit(1)
            elif a.mode == "hang":
                print(f"rank {rank}: hanging on purpose", flush=True)
                time.sleep(3600)
            else:
                print(f"rank {rank}: exiting on purpose", flush=True)
                os._exit(0)
        idx = torch.randint(0, 512, (2, 64), generator=g)
        opt.zero_grad()
        _, loss = model(idx, idx)
        loss.backward()
        allreduce_gradients(model, dp)
        opt.step()
        hb.tick()
    hb.stop()
    wd.stop()
    dist.destroy_process_group()
    sys.exit(0)


if __name__ == "__main__":
    main()
