"""Data parallelism composed with TP, PP, interleaving and SP.

    python -m dstraining_b200.utils.launch 8 tests/suites/dp_suite.py --dp 2 --pp 2 --tp 2 --chunks 2 --micro 1 --sp --bucketed

Each replica takes its slice of the global batch. Checks (fp32, against the
full model on the FULL global batch): DP-averaged gradients; the DP-averaged
loss; a 5-step Adam trajectory that falls. ``--bucketed`` uses
``GradReducer`` with 256 KiB buckets so many buckets are exercised.
Mirrors the reference suite ``tests/test_dp_correctness.py``.
"""

import argparse

from common import ATOL, SEED, Report, batch, small_config, start, worst_grad

import torch
import torch.distributed as dist

from dstraining_b200.models.gpt import GPT, GPTChunks, GPTStage
from dstraining_b200.parallel import topology
from dstraining_b200.parallel.dp import GradReducer, allreduce_gradients
from dstraining_b200.parallel.pipeline import Pipeline1F1B, PipelineInterleaved


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--pp", type=int, default=1)
    ap.add_argument("--dp", type=int, default=2)
    ap.add_argument("--micro", type=int, default=1)
    ap.add_argument("--sp", action="store_true")
    ap.add_argument("--chunks", type=int, default=1)
    ap.add_argument("--bucketed", action="store_true")
    ap.add_argument("--device", default=None)
    a = ap.parse_args()
    device = start(a.device)
    tp, pp, dp = topology.make_topology(a.tp, a.pp, a.dp)
    rep = Report()
    cfg = small_config(sequence_parallel=a.sp)
    B, b = 8, 8 // a.dp
    rep.say(f"dp={a.dp} tp={a.tp} pp={a.pp} chunks={a.chunks} sp={a.sp} bucketed={a.bucketed}")

    ref = GPT(cfg, topology.SINGLE, seed=SEED).to(device)
    if a.chunks > 1:
        model = GPTChunks(cfg, tp, pp, v=a.chunks, seed=SEED).to(device)
        pipe = PipelineInterleaved(model, pp, micro_batch_size=a.micro, seq_len=cfg.block_size)
    elif a.pp > 1:
        model = GPTStage(cfg, tp, pp, seed=SEED).to(device)
        pipe = Pipeline1F1B(model, pp, micro_batch_size=a.micro, seq_len=cfg.block_size)
    else:
        model = GPT(cfg, tp, seed=SEED).to(device)
        pipe = None
    idx, tgt = batch(cfg, B, SEED + 1, device)
    my_idx, my_tgt = idx[dp.rank * b : (dp.rank + 1) * b], tgt[dp.rank * b : (dp.rank + 1) * b]
    reducer = GradReducer(model, dp, bucket_bytes=1 << 18, overlap=pipe is None) if a.bucketed else None

    def step():
        model.zero_grad(set_to_none=True)
        if pipe is not None:
            loss = pipe.train_step(my_idx, my_tgt)
            if reducer is not None:
                reducer.reduce()
        else:
            _, loss = model(my_idx, my_tgt)
            loss.backward()
        if reducer is not None:
            reducer.finish()
        else:
            allreduce_gradients(model, dp)
        model.finalize_grads()
        if pp.is_last:
            avg = loss.detach().clone()
            dist.all_reduce(avg, group=dp.group)
            return avg / dp.world
        return None

    loss = step()
    _, loss_ref = ref(idx, tgt)
    loss_ref.backward()
    name, worst = worst_grad(model, ref, tp, model.ref_param_name)
    rep.close(f"DP-averaged grads (worst {name})", worst)
    if pp.is_last:
        d = abs(loss.item() - loss_ref.item())
        rep.ok &= d <= ATOL
        if tp.rank == 0 and dp.rank == 0:
            print(f"  [{'PASS' if d <= ATOL else 'FAIL'}] DP-averaged loss: max abs diff {d:.3e}", flush=True)

    opt = torch.optim.Adam(model.parameters(), lr=1e-3)
    opt_ref = torch.optim.Adam(ref.parameters(), lr=1e-3)
    ref.zero_grad(set_to_none=True)
    losses, worst = [], 0.0
    for _ in range(5):
        loss = step()
        opt.step()
        opt_ref.zero_grad(set_to_none=True)
        _, loss_ref = ref(idx, tgt)
        loss_ref.backward()
        opt_ref.step()
        if pp.is_last:
            worst = max(worst, abs(loss.item() - loss_ref.item()))
            losses.append(loss.item())
    if pp.is_last:
        good = worst <= 1e-4 and losses[-1] < losses[0]
        rep.ok &= good
        if tp.rank == 0 and dp.rank == 0:
            print(f"  [{'PASS' if good else 'FAIL'}] 5-step trajectory diff {worst:.3e}, "
                  f"loss {losses[0]:.4f} -> {losses[-1]:.4f}", flush=True)
    rep.finish(device)


if __name__ == "__main__":
    main()
