"""bf16 + fp32 master weights.

    python -m dstraining_b200.utils.launch 2 tests/suites/precision_suite.py

Over 30 steps on a fixed batch: bf16 + masters trains (loss falls by > 1.0)
and lands within 0.3 of the fp32 run; plain bf16 Adam (updates rounded to
bf16 every step) ends measurably worse (> 0.05); parameters stay bf16 and
bitwise equal to ``master.to(bf16)``, masters and Adam moments stay fp32;
under TP the bf16 logits are bitwise identical across ranks. Mirrors
``tests/test_precision.py`` of the reference. With ``--device cuda`` the
bf16 runs take the native kernels (fused Adam included).
"""

import argparse

from common import SEED, Report, small_config, start

import torch
import torch.distributed as dist

from dstraining_b200.models.gpt import GPT
from dstraining_b200.optim.precision import MasterWeightOptimizer
from dstraining_b200.parallel import topology

STEPS = 30


def train(model, opt, idx, tgt):
    out = []
    for _ in range(STEPS):
        opt.zero_grad(set_to_none=True)
        _, loss = model(idx, tgt)
        loss.backward()
        model.finalize_grads()
        opt.step()
        out.append(loss.item())
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--device", default=None)
    a = ap.parse_args()
    device = start(a.device)
    tp = topology.make_tp_context()
    rep = Report()
    cfg = small_config()
    g = torch.Generator().manual_seed(SEED + 1)
    idx = torch.randint(0, cfg.vocab_size, (4, cfg.block_size), generator=g).to(device)
    tgt = torch.randint(0, cfg.vocab_size, (4, cfg.block_size), generator=g).to(device)
    rep.say(f"tp={tp.world}, {STEPS} steps")

    m32 = GPT(cfg, tp, seed=SEED).to(device)
    fp32 = train(m32, torch.optim.Adam(m32.parameters(), lr=1e-3), idx, tgt)
    m16 = GPT(cfg, tp, seed=SEED).to(device).to(torch.bfloat16)
    opt = MasterWeightOptimizer(m16.parameters(), lr=1e-3)
    bf16 = train(m16, opt, idx, tgt)
    bad_model = GPT(cfg, tp, seed=SEED).to(device).to(torch.bfloat16)
    bad = train(bad_model, torch.optim.Adam(bad_model.parameters(), lr=1e-3), idx, tgt)

    rep.flag(f"bf16+masters trains {bf16[0]:.4f} -> {bf16[-1]:.4f} (fp32 {fp32[0]:.4f} -> {fp32[-1]:.4f})",
             bf16[-1] < bf16[0] - 1.0)
    rep.flag(f"tracks fp32: final gap {abs(bf16[-1] - fp32[-1]):.4f} < 0.3", abs(bf16[-1] - fp32[-1]) < 0.3)
    rep.flag(f"plain bf16 Adam ends worse: {bad[-1]:.4f} vs {bf16[-1]:.4f}", bad[-1] > bf16[-1] + 0.05)
    dtypes = all(p.dtype == torch.bfloat16 for p in m16.parameters())
    dtypes &= all(m.dtype == torch.float32 for m in opt.master_params)
    dtypes &= all(s["exp_avg"].dtype == torch.float32 for s in opt.inner.state.values())
    synced = all(torch.equal(p.data, m.to(torch.bfloat16)) for p, m in zip(opt.model_params, opt.master_params))
    rep.flag("params bf16 == master.to(bf16); masters and moments fp32", dtypes and synced)
    if tp.enabled:
        logits, _ = m16(idx, tgt)
        parts = [torch.empty_like(logits) for _ in range(tp.world)]
        dist.all_gather(parts, logits.detach().contiguous(), group=tp.group)
        d = max((p.float() - parts[0].float()).abs().max().item() for p in parts)
        rep.close("cross-rank bf16 logit identity", d, atol=0.0)
    rep.finish(device)


if __name__ == "__main__":
    main()
