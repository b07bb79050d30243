"""Gradient accumulation without pipelining (``Trainer`` with --grad-accum):
a batch of 8 in micro-batches of 2 must train exactly like the batch in one
piece (fp32, CPU), with data parallelism over the ranks - the DP reducer's
hooks must wait for the last micro-batch. The fused DP optimizer's hook
deferral is checked the same way through its emulated (gloo) path.

    python -m dstraining_b200.utils.launch 2 tests/suites/accum_suite.py
"""

import argparse

from common import Report, start

import torch
import torch.distributed as dist

from dstraining_b200.optim.fused_dp import FusedDPAdam
from dstraining_b200.trainer import Trainer, add_args


def run(extra, steps=3):
    argv = ["--dp", str(dist.get_world_size()), "--layers", "2", "--heads", "4", "--embd", "64", "--block", "32",
            "--vocab", "256", "--batch", "8", "--device", "cpu", "--seed", "7", *extra]
    tr = Trainer(add_args(argparse.ArgumentParser()).parse_args(argv))
    out = []
    for s in range(steps):
        x, y = tr.shard.get_batch(s)
        out.append(tr.step_device(x, y).item())
    return tr, out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--device", default="cpu")
    a = ap.parse_args()
    device = start(a.device)
    rep = Report()
    whole, l1 = run([])
    accum, l2 = run(["--grad-accum", "--micro", "2"])
    rep.flag("accumulation active", accum.accum == 4 and whole.accum == 1)
    rep.close("losses: micro-batches 4 x 2 vs batch 8", max(abs(x - y) for x, y in zip(l1, l2)), atol=1e-5)
    worst = max((p.data - q.data).abs().max().item()
                for p, q in zip(whole.model.parameters(), accum.model.parameters()))
    rep.close("parameters after 3 steps", worst, atol=1e-5)

    # Fused DP optimizer (emulated path): deferred hooks, then one launch per bucket.
    torch.manual_seed(0)
    ref_tr, _ = run([], steps=0)
    acc_tr, _ = run([], steps=0)
    for tr in (ref_tr, acc_tr):
        tr.opt = FusedDPAdam(tr.model, tr.dp, lr=3e-4, bucket_bytes=1 << 14)
        tr.reducer = None
        tr.fused_dp = True
    acc_tr.accum, acc_tr.args.micro = 4, 2
    for s in range(2):
        x, y = ref_tr.shard.get_batch(s)
        ref_tr.step_device(x, y)
        acc_tr.step_device(x, y)
    worst = max((p.data - q.data).abs().max().item()
                for p, q in zip(ref_tr.model.parameters(), acc_tr.model.parameters()))
    rep.close("fused DP optimizer with deferred hooks: parameters", worst, atol=1e-5)
    rep.finish(device)


if __name__ == "__main__":
    main()
