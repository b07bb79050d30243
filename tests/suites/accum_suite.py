"""Gradient accumulation without pipelining (``Trainer`` with --grad-accum):
a batch of 8 in micro-batches of 2 must train exactly like the batch in one
piece (fp32, CPU), with data parallelism over the ranks - the DP reducer's
hooks must wait for the last micro-batch. The fused DP optimizer's hook
deferral is checked the same way through its emulated (gloo) path.

    python -m dstraining_b200.utils.launch 2 tests/suites/accum_suite.py
"""

import argparse

from common import NoiseLevelGrads, Report, start

import torch
import torch.distributed as dist

from dstraining_b200.optim.fused_dp import FusedDPAdam
from dstraining_b200.trainer import Trainer, add_args


def run(extra, steps=3, noisy=None):
    argv = ["--dp", str(dist.get_world_size()), "--layers", "2", "--heads", "4", "--embd", "64", "--block", "32",
            "--vocab", "256", "--batch", "8", "--device", "cpu", "--seed", "7", *extra]
    tr = Trainer(add_args(argparse.ArgumentParser()).parse_args(argv))
    out = []
    for s in range(steps):
        x, y = tr.shard.get_batch(s)
        out.append(tr.step_device(x, y).item())
        if noisy is not None:
            noisy.record(tr.model)
    return tr, out


def params_close(rep, name, ref_tr, tr, noisy, lr, steps):
    """Parameters of two runs: 1e-5, except elements whose gradient was at
    the rounding-noise level, held to Adam's bound of lr per step."""
    worst, worst_noisy, n_noisy = noisy.compare(
        (n, q.data, p.data) for (n, p), q in zip(ref_tr.model.named_parameters(), tr.model.parameters()))
    rep.close(name, worst, atol=1e-5)
    rep.close(f"{name} with a noise-level gradient ({n_noisy} elements) within steps x lr", worst_noisy,
              atol=steps * lr)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--device", default="cpu")
    a = ap.parse_args()
    device = start(a.device)
    rep = Report()
    noisy = NoiseLevelGrads()
    whole, l1 = run([], noisy=noisy)
    accum, l2 = run(["--grad-accum", "--micro", "2"])
    rep.flag("accumulation active", accum.accum == 4 and whole.accum == 1)
    rep.close("losses: micro-batches 4 x 2 vs batch 8", max(abs(x - y) for x, y in zip(l1, l2)), atol=1e-5)
    params_close(rep, "parameters after 3 steps", whole, accum, noisy, lr=3e-4, steps=3)

    # Fused DP optimizer (emulated path): deferred hooks, then one launch per bucket.
    torch.manual_seed(0)
    ref_tr, _ = run([], steps=0)
    acc_tr, _ = run([], steps=0)
    for tr in (ref_tr, acc_tr):
        tr.opt = FusedDPAdam(tr.model, tr.dp, lr=3e-4, bucket_bytes=1 << 14)
        tr.reducer = None
        tr.fused_dp = True
    acc_tr.accum, acc_tr.args.micro = 4, 2
    noisy = NoiseLevelGrads()
    for s in range(2):
        x, y = ref_tr.shard.get_batch(s)
        ref_tr.step_device(x, y)
        noisy.record(ref_tr.model)
        acc_tr.step_device(x, y)
    params_close(rep, "fused DP optimizer with deferred hooks: parameters", ref_tr, acc_tr, noisy, lr=3e-4, steps=2)
    rep.finish(device)


if __name__ == "__main__":
    main()
