"""Fused DP reduce + Adam (FusedDPAdam) against references.

    python -m dstraining_b200.utils.launch 2 tests/suites/fused_dp_suite.py --dp 2
    torchrun --nproc-per-node 2 tests/suites/fused_dp_suite.py --dp 2 --device cuda --bf16

fp32 (CPU: the host transport, or ``--transport collectives``, the sharded
reduce-scatter / all-gather path that DP groups spanning machines use on
GPUs): every rank trains its slice of the global batch
with FusedDPAdam; the loss trajectory and final weights must match a
single-process model trained with torch.optim.Adam on the full batch.
bf16 on CUDA (the native NVLink kernel): the same run must track the unfused
path (bucketed all-reduce + MasterWeightOptimizer) on identical data within
bf16 rounding, and parameters must stay identical across DP ranks.
"""

import argparse

from common import SEED, NoiseLevelGrads, Report, batch, max_diff, small_config, start

import torch
import torch.distributed as dist

from dstraining_b200.models.gpt import GPT
from dstraining_b200.optim.fused_dp import FusedDPAdam
from dstraining_b200.optim.precision import MasterWeightOptimizer
from dstraining_b200.parallel import topology
from dstraining_b200.parallel.dp import GradReducer


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--dp", type=int, default=2)
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--sp", action="store_true")
    ap.add_argument("--bf16", action="store_true")
    ap.add_argument("--device", default=None)
    ap.add_argument("--transport", default="auto", help="FusedDPAdam transport (auto, peer, collectives, host)")
    a = ap.parse_args()
    device = start(a.device)
    tp, pp, dp = topology.make_topology(a.tp, 1, a.dp)
    rep = Report()
    # the native attention kernels take head_dim 64 or 128
    cfg = small_config(sequence_parallel=a.sp, block_size=128 if a.bf16 else 64, n_embd=128,
                       n_head=2 if a.bf16 else 8)
    B, steps = 8, 4
    b = B // dp.world
    dtype = torch.bfloat16 if a.bf16 else torch.float32
    rep.say(f"dp={a.dp} tp={a.tp} sp={a.sp} dtype={dtype} device={device}")

    def build():
        m = GPT(cfg, tp, seed=SEED).to(device)
        return m.to(dtype)

    model = build()
    opt = FusedDPAdam(model, dp, lr=1e-3, bucket_bytes=1 << 16, transport=a.transport)
    rep.say(f"transport {opt.transport}")
    rep.flag(f"{len(opt.buckets)} buckets", len(opt.buckets) > 2)
    if a.bf16:
        ref = build()
        ref_opt = MasterWeightOptimizer(ref.parameters(), lr=1e-3)
        reducer = GradReducer(ref, dp, bucket_bytes=1 << 16)
    else:
        ref = GPT(cfg, topology.SINGLE, seed=SEED).to(device)
        ref_opt = torch.optim.Adam(ref.parameters(), lr=1e-3)
    worst_loss = 0.0
    noisy = NoiseLevelGrads()  # fp32: reference elements with a noise-level gradient
    for s in range(steps):
        idx, tgt = batch(cfg, B, SEED + 10 + s, device)
        mine = slice(dp.rank * b, (dp.rank + 1) * b)
        opt.zero_grad()
        _, loss = model(idx[mine], tgt[mine])
        loss.backward()
        model.finalize_grads()
        opt.step()
        ref_opt.zero_grad(set_to_none=True)
        if a.bf16:
            _, rl = ref(idx[mine], tgt[mine])
            rl.backward()
            reducer.finish()
            ref.finalize_grads()
        else:
            _, rl = ref(idx, tgt)
            rl.backward()
        if not a.bf16:
            noisy.record(ref)
        ref_opt.step()
        lm = loss.detach().float().clone()
        dist.all_reduce(lm, group=dp.group)
        rlm = rl.detach().float().clone()
        if a.bf16:
            dist.all_reduce(rlm, group=dp.group)
            rlm /= dp.world
        worst_loss = max(worst_loss, abs(lm.item() / dp.world - rlm.item()))
    rep.close("loss trajectory vs reference", worst_loss, atol=2e-2 if a.bf16 else 1e-5)
    ref_p = dict(ref.named_parameters())
    pairs = [(name, p.data, ref_p[name].data) for name, p in model.named_parameters()
             if a.bf16 or p.shape == ref_p[name].shape]  # TP shards vs full reference: covered by the loss check
    worst, worst_noisy, n_noisy = noisy.compare(pairs)
    rep.close("final parameters vs reference", worst, atol=2e-2 if a.bf16 else 1e-4)
    if not a.bf16:
        rep.close(f"final parameters with a noise-level gradient ({n_noisy} elements) within steps x lr", worst_noisy,
                  atol=steps * 1e-3)
    # replicas must hold bitwise-identical parameters
    flat = torch.cat([p.data.float().reshape(-1) for p in model.parameters()])
    parts = [torch.empty_like(flat) for _ in range(dp.world)]
    dist.all_gather(parts, flat, group=dp.group)
    rep.close("parameters identical across DP ranks", max(max_diff(x, parts[0]) for x in parts), atol=0.0)
    if device.type == "cuda":
        from dstraining_b200.ops import native

        errs = opt.protocol_errors()
        rep.flag(f"signal protocol invariants {errs or 'hold'}", not errs, only_rank0=False)
        rep.flag("device status word clear", native.lib().read_status(True) == 0, only_rank0=False)
    rep.finish(device)


if __name__ == "__main__":
    main()
