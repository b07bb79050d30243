"""Sharded checkpoint round trip and resharding.

    python -m dstraining_b200.utils.launch 4 tests/suites/ckpt_suite.py --tp 2 --pp 2 --dir /tmp/ck

Checks (fp32, Adam): training N steps straight equals training k steps,
saving, rebuilding everything from a different seed, loading, and training
the remaining steps (bitwise-equal losses); the checkpoint written at this
rank's tp/pp loads into a single-process tp=1 model (rank 0), whose loss on
the next batch matches the parallel model's.
"""

import argparse
import shutil

from common import Report, start

import torch
import torch.distributed as dist

from dstraining_b200.models.gpt import GPT
from dstraining_b200.parallel import topology
from dstraining_b200.trainer import Trainer, add_args
from dstraining_b200.utils import checkpoint


def trainer(tp, pp, seed, micro):
    a = add_args(argparse.ArgumentParser()).parse_args(
        ["--device", "cpu", "--tp", str(tp), "--pp", str(pp), "--layers", "4", "--batch", "4", "--micro", str(micro),
         "--lr", "1e-3", "--seed", str(seed)]
    )
    return Trainer(a)


def losses(tr, steps, first):
    out = []
    for s in range(first, first + steps):
        idx, tgt = tr.shard.get_batch(s)
        loss = tr.step_device(idx, tgt)
        out.append(None if loss is None else loss.item())
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tp", type=int, default=2)
    ap.add_argument("--pp", type=int, default=1)
    ap.add_argument("--dir", required=True)
    ap.add_argument("--device", default="cpu")
    ap.add_argument("--background", action="store_true", help="write the checkpoint from a thread")
    a = ap.parse_args()
    device = start(a.device)
    rep = Report()
    micro = 2 if a.pp > 1 else 1
    if dist.get_rank() == 0:
        shutil.rmtree(a.dir, ignore_errors=True)
    dist.barrier()

    ref = trainer(a.tp, a.pp, seed=11, micro=micro)
    straight = losses(ref, 6, 0)

    tr = trainer(a.tp, a.pp, seed=11, micro=micro)
    first = losses(tr, 3, 0)
    if a.background:
        pending = checkpoint.save(a.dir, 3, tr.model, tr.opt, tr.tp, tr.pp, tr.dp, tr.config, 11, background=True)
        losses(tr, 2, 3)  # keep training while the files are written: the snapshot must not change
        path = pending.wait()
        dist.barrier()
        rep.flag("background save marked complete", checkpoint.latest(a.dir) == path)
    else:
        path = checkpoint.save(a.dir, 3, tr.model, tr.opt, tr.tp, tr.pp, tr.dp, tr.config, 11)
    del tr
    tr2 = trainer(a.tp, a.pp, seed=11, micro=micro)  # same data stream
    with torch.no_grad():  # scramble the weights: the load must overwrite all of them
        for p in tr2.model.parameters():
            p.normal_()
    checkpoint.load(path, tr2.model, tr2.opt, tr2.tp)
    resumed = first + losses(tr2, 3, 3)
    if tr2.pp.is_last:
        same = all(x == y for x, y in zip(straight, resumed))
        rep.ok &= same
        if tr2.tp.rank == 0:
            print(f"  [{'PASS' if same else 'FAIL'}] resume: {straight} == {resumed}", flush=True)

    # Reshard: rank 0 loads the checkpoint into a single-process tp=1 model.
    next_loss = None
    if dist.get_rank() == 0:
        m1 = GPT(tr2.config, topology.SINGLE, seed=12345)
        checkpoint.load(path, m1, None, topology.SINGLE)
        idx, tgt = tr2.shard.get_batch(3)
        with torch.no_grad():
            _, next_loss = m1(idx, tgt)
        d = abs(next_loss.item() - straight[3]) if straight[3] is not None else 0.0
        # rank 0 is the first stage; compare against the value broadcast below
    val = torch.tensor([straight[3] if straight[3] is not None else 0.0])
    src = dist.get_world_size() - 1  # last stage holds the loss
    dist.broadcast(val, src=src)
    if dist.get_rank() == 0:
        d = abs(next_loss.item() - val.item())
        rep.close("tp1 model loaded from the sharded checkpoint: next-step loss", d, only_rank0=False)
    rep.finish(device)


if __name__ == "__main__":
    main()
