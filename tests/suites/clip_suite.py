"""Global gradient norm under TP (+SP): equals the single-process model's
norm on the same batch (shards counted by shard, replicated parameters once).

    python -m dstraining_b200.utils.launch 2 tests/suites/clip_suite.py --sp
"""

import argparse
from dataclasses import replace

from common import SEED, Report, batch, small_config, start

import torch

from dstraining_b200.models.gpt import GPT
from dstraining_b200.optim.clip import clip_grad_norm, grad_norm
from dstraining_b200.parallel import topology


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--sp", action="store_true")
    ap.add_argument("--device", default="cpu")
    a = ap.parse_args()
    device = start(a.device)
    import torch.distributed as dist

    tp, _, dp = topology.make_topology(dist.get_world_size(), 1, 1)
    cfg = replace(small_config(), sequence_parallel=a.sp)
    rep = Report()
    model = GPT(cfg, tp, seed=SEED).to(device)
    ref = GPT(replace(cfg, sequence_parallel=False), topology.SINGLE, seed=SEED).to(device)
    idx, tgt = batch(cfg, 4, SEED + 1, device)
    for m in (model, ref):
        _, loss = m(idx, tgt)
        loss.backward()
    model.finalize_grads()
    want = torch.sqrt(sum(p.grad.double().pow(2).sum() for p in ref.parameters())).item()
    got = grad_norm(model, tp, dp).item()
    rep.close("global gradient norm vs single-process model", abs(got - want) / want, atol=1e-5)
    norm = clip_grad_norm(model, 0.5 * want, tp, dp)
    after = grad_norm(model, tp, dp).item()
    rep.close("norm after clipping to half", abs(after - 0.5 * want) / want, atol=1e-4)
    rep.flag("clip returns the norm before clipping", abs(norm - want) / want < 1e-5)
    rep.finish(device)


if __name__ == "__main__":
    main()
