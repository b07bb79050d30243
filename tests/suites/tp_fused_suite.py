"""Fused tensor-parallel kernels (AG+GEMM, GEMM+RS over NVLink) vs tp=1.

    torchrun --nproc-per-node 2 tests/suites/tp_fused_suite.py --sp
    torchrun --nproc-per-node 2 tests/suites/tp_fused_suite.py [--nccl-mlp]

bf16 on CUDA. Every rank builds the TP model and the single-GPU model with
identical weights (decomposition-invariant init). Checks: the loss matches;
every gradient shard matches the corresponding slice of the single-GPU
gradient (after finalize_grads); the loss is identical on every rank; three
optimizer steps keep the two in step; the device status word stays clear.
"""

import argparse

from common import SEED, Report, batch, max_diff, shard_of, start

import torch
import torch.distributed as dist

from dstraining_b200.models.gpt import GPT, GPTConfig
from dstraining_b200.ops import native
from dstraining_b200.optim.precision import MasterWeightOptimizer
from dstraining_b200.parallel import topology


def rel(a, b):
    return (a.float() - b.float()).abs().max().item() / max(b.float().abs().max().item(), 1e-6)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--sp", action="store_true")
    ap.add_argument("--device", default="cuda")
    ap.add_argument("--nccl-mlp", action="store_true",
                    help="without --sp: the MLP with NCCL all-reduces around the native GEMMs (DST_FUSED_TP_MLP=0) "
                    "instead of the fused replicated-activation form")
    a = ap.parse_args()
    if a.nccl_mlp:
        import os

        os.environ["DST_FUSED_TP_MLP"] = "0"
    device = start(a.device)
    tp = topology.make_tp_context()
    rep = Report()
    cfg = GPTConfig(vocab_size=1000, block_size=128 * tp.world, n_layer=2, n_head=2 * tp.world, n_embd=128 * tp.world,
                    sequence_parallel=a.sp, vocab_parallel_loss=True)
    rep.say(f"tp={tp.world} sp={a.sp} T={cfg.block_size} C={cfg.n_embd}")
    model = GPT(cfg, tp, seed=SEED).to(device).to(torch.bfloat16)
    ref = GPT(cfg, topology.SINGLE, seed=SEED).to(device).to(torch.bfloat16)
    idx, tgt = batch(cfg, 2, SEED + 1, device)

    _, loss = model(idx, tgt)
    _, loss_ref = ref(idx, tgt)
    rep.close("loss vs tp=1", abs(loss.item() - loss_ref.item()), atol=2e-2)
    parts = [torch.empty(1, device=device) for _ in range(tp.world)]
    dist.all_gather(parts, loss.detach().float().reshape(1), group=tp.group)
    rep.close("loss identical across ranks", max(max_diff(p, parts[0]) for p in parts), atol=0.0)
    loss.backward()
    model.finalize_grads()
    loss_ref.backward()
    ref_p = dict(ref.named_parameters())
    worst, worst_name = 0.0, None
    for name, p in model.named_parameters():
        r = rel(p.grad, shard_of(model, name, p, ref_p[name].grad, tp))
        if r > worst:
            worst, worst_name = r, name
    rep.close(f"all grad shards vs tp=1 (relative, worst {worst_name})", worst, atol=6e-2)

    opt = MasterWeightOptimizer(model.parameters(), lr=1e-3)
    opt_ref = MasterWeightOptimizer(ref.parameters(), lr=1e-3)
    traj = 0.0
    for s in range(3):
        idx, tgt = batch(cfg, 2, SEED + 10 + s, device)
        for m, o in ((model, opt), (ref, opt_ref)):
            o.zero_grad()
            _, l_ = m(idx, tgt)
            l_.backward()
            m.finalize_grads()
            o.step()
            if m is model:
                lm = l_.item()
            else:
                lr_ = l_.item()
        traj = max(traj, abs(lm - lr_))
    rep.close("3-step trajectory vs tp=1", traj, atol=3e-2)
    rep.flag("device status word clear", native.lib().read_status(True) == 0, only_rank0=False)
    rep.finish(device)


if __name__ == "__main__":
    main()
