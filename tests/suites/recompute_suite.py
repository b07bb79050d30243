"""Selective recompute: bitwise equivalence, memory drop, call count.

    python tests/suites/recompute_suite.py

Single process. Checks: with recompute on, logits, loss and every gradient
are bitwise equal to the run without it; the bytes autograd saves for
backward (counted with ``saved_tensors_hooks``) drop by at least the
``2 * s^2 * b * a * 4 * L`` attention-matrix term; the recomputed region is
entered once per layer in forward. Mirrors ``tests/test_recompute.py`` of the
reference.
"""

import sys

from common import SEED, small_config

import torch

from dstraining_b200.models.gpt import GPT
from dstraining_b200.ops import recompute as rc
from dstraining_b200.parallel import topology


def run(cfg, idx, tgt):
    model = GPT(cfg, topology.SINGLE, seed=SEED)
    saved = 0

    def pack(t):
        nonlocal saved
        saved += t.nbytes
        return t

    with torch.autograd.graph.saved_tensors_hooks(pack, lambda t: t):
        logits, loss = model(idx, tgt)
    loss.backward()
    return logits.detach(), loss.detach(), {n: p.grad.clone() for n, p in model.named_parameters()}, saved


def main():
    B, s, a, L = 4, 64, 8, 4
    g = torch.Generator().manual_seed(SEED + 1)
    idx = torch.randint(0, 512, (B, s), generator=g)
    tgt = torch.randint(0, 512, (B, s), generator=g)
    entries = 0
    original = rc._Recompute.forward

    def counted(ctx, fn, *args):
        nonlocal entries
        entries += 1
        return original(ctx, fn, *args)

    rc._Recompute.forward = staticmethod(counted)
    l0, loss0, g0, b0 = run(small_config(), idx, tgt)
    l1, loss1, g1, b1 = run(small_config(recompute_attention=True), idx, tgt)
    rc._Recompute.forward = staticmethod(original)

    ok = True
    exact = torch.equal(l0, l1) and torch.equal(loss0, loss1) and all(torch.equal(g0[n], g1[n]) for n in g0)
    ok &= exact
    print(f"  [{'PASS' if exact else 'FAIL'}] bitwise equal logits, loss and all grads")
    term = 2 * (B * a * s * s) * 4 * L
    drop = b0 - b1
    ok &= drop >= term
    print(f"  [{'PASS' if drop >= term else 'FAIL'}] saved bytes {b0:,} -> {b1:,} (dropped {drop:,} >= {term:,})")
    ok &= entries == L
    print(f"  [{'PASS' if entries == L else 'FAIL'}] region entered {entries} times in forward (L={L})")
    print("\nALL PASS" if ok else "\nFAILED")
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
