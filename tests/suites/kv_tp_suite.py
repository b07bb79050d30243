"""KV-cache decoding of a tensor-parallel GPT against the single-process model.

    python -m dstraining_b200.utils.launch 2 tests/suites/kv_tp_suite.py

Every rank builds the TP model and the tp=1 model with identical weights
(decomposition-invariant init). Checks: the cached decoder's logits for a
prompt and each following token equal the tp=1 full forward pass's, and
greedy generation through the cache (also past block_size, where the window
slides) gives the tp=1 tokens on every rank.
"""

import argparse

from common import SEED, Report, max_diff, small_config, start

import torch
import torch.distributed as dist

from dstraining_b200.models.gpt import GPT
from dstraining_b200.parallel import topology
from dstraining_b200.utils.generate import KVCache, generate


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--device", default=None)
    a = ap.parse_args()
    device = start(a.device)
    tp = topology.make_tp_context()
    rep = Report()
    cfg = small_config(block_size=32, n_layer=2, n_head=4, n_embd=64, vocab_size=300)
    model = GPT(cfg, tp, seed=SEED).to(device).eval()
    ref = GPT(cfg, topology.SINGLE, seed=SEED).to(device).eval()
    seq = torch.randint(0, 300, (2, 24), generator=torch.Generator().manual_seed(SEED + 1)).to(device)
    cache = KVCache(model, 2)
    with torch.no_grad():
        got = [cache.forward(seq[:, :7])] + [cache.forward(seq[:, t : t + 1]) for t in range(7, 24)]
        want = ref(seq)[0][:, 6:, :300]
    rep.close("cached TP logits vs tp=1 full forward", max_diff(torch.stack(got, 1), want), atol=2e-5)
    out = generate(model, seq[:, :5], 40, temperature=0.0)  # 45 > block_size: the window slides
    out_ref = generate(ref, seq[:, :5], 40, temperature=0.0, use_cache=False, pad_to=1)
    rep.flag("greedy tokens equal tp=1", torch.equal(out, out_ref), only_rank0=False)
    parts = [torch.empty_like(out) for _ in range(tp.world)]
    dist.all_gather(parts, out, group=tp.group)
    rep.flag("tokens identical on every rank", all(torch.equal(p, parts[0]) for p in parts))
    rep.finish(device)


if __name__ == "__main__":
    main()
