"""Pipeline (1F1B / interleaved) correctness, composed with TP/SP.

    python -m dstraining_b200.utils.launch 4 tests/suites/pp_suite.py --pp 2 --tp 2 --chunks 2 --micro 1 --sp

Checks (fp32): the microbatched pipeline loss equals the full-batch loss;
gradients accumulated over microbatches match the full model's; a 5-step
Adam trajectory tracks the full model and falls; the interleaved schedule's
peak number of stashed activations stays within its warm-up depth + 1.
Mirrors the reference suite ``tests/test_pp_correctness.py``.
"""

import argparse

from common import ATOL, SEED, Report, batch, small_config, start, worst_grad

import torch

from dstraining_b200.models.gpt import GPT, GPTChunks, GPTStage
from dstraining_b200.parallel import topology
from dstraining_b200.parallel.pipeline import Pipeline1F1B, PipelineInterleaved


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--pp", type=int, default=2)
    ap.add_argument("--micro", type=int, default=1)
    ap.add_argument("--sp", action="store_true")
    ap.add_argument("--chunks", type=int, default=1)
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--device", default=None)
    a = ap.parse_args()
    device = start(a.device)
    tp, pp, _ = topology.make_topology(a.tp, a.pp)
    rep = Report()
    cfg = small_config(n_layer=a.layers, sequence_parallel=a.sp)
    B = 4
    m = B // a.micro
    rep.say(f"tp={a.tp} pp={a.pp} chunks={a.chunks} sp={a.sp} layers={a.layers} microbatches={m}")

    ref = GPT(cfg, topology.SINGLE, seed=SEED).to(device)
    if a.chunks > 1:
        stage = GPTChunks(cfg, tp, pp, v=a.chunks, seed=SEED).to(device)
        pipe = PipelineInterleaved(stage, pp, micro_batch_size=a.micro, seq_len=cfg.block_size)
    else:
        stage = GPTStage(cfg, tp, pp, seed=SEED).to(device)
        pipe = Pipeline1F1B(stage, pp, micro_batch_size=a.micro, seq_len=cfg.block_size)
    idx, tgt = batch(cfg, B, SEED + 1, device)
    last_tp0 = pp.is_last and tp.rank == 0

    stage.zero_grad(set_to_none=True)
    loss = pipe.train_step(idx, tgt)
    stage.finalize_grads()
    _, loss_ref = ref(idx, tgt)
    loss_ref.backward()
    if pp.is_last:
        rep.close("pipelined loss vs full batch", abs(loss.item() - loss_ref.item()), only_rank0=False) if last_tp0 else None
        rep.ok &= abs(loss.item() - loss_ref.item()) <= ATOL
    else:
        rep.flag("non-last stage returns no loss", loss is None, only_rank0=False)
    name, worst = worst_grad(stage, ref, tp, stage.ref_param_name)
    rep.close(f"accumulated grads (worst {name})", worst)

    opt = torch.optim.Adam(stage.parameters(), lr=1e-3)
    opt_ref = torch.optim.Adam(ref.parameters(), lr=1e-3)
    losses, worst = [], 0.0
    for _ in range(5):
        opt.zero_grad(set_to_none=True)
        loss = pipe.train_step(idx, tgt)
        stage.finalize_grads()
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
        if last_tp0:
            print(f"  [{'PASS' if worst <= 1e-4 else 'FAIL'}] 5-step trajectory: max abs diff {worst:.3e}", flush=True)
            print(f"  [{'PASS' if losses[-1] < losses[0] else 'FAIL'}] loss falls {losses[0]:.4f} -> {losses[-1]:.4f}", flush=True)
    if a.chunks > 1:
        bound = min(2 * (a.pp - 1 - pp.rank) + (a.chunks - 1) * a.pp, m * a.chunks) + 1
        rep.flag(f"rank0 peak in-flight {pipe.peak_in_flight} <= warm-up + 1 = {bound}", pipe.peak_in_flight <= bound)
    rep.finish(device)


if __name__ == "__main__":
    main()
