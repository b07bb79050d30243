"""Tensor (+sequence) parallel correctness, TP degree = world size.

    python -m dstraining_b200.utils.launch 2 tests/suites/tp_suite.py --sp --recompute --vp

Checks (fp32, against the single-process model with identical weights):
conjugacy of f/f̄ (and g/ḡ with --sp) on a toy split MLP; LayerNorm inputs
sequence-sharded under SP; every shard is an exact slice of the full
weights; logits and loss match and logits are bitwise identical across
ranks; every gradient matches; 10 Adam steps track the full model and the
loss falls. Mirrors the reference suite ``tests/test_tp_correctness.py``.
"""

import argparse
from dataclasses import replace

from common import SEED, Report, batch, max_diff, shard_of, small_config, start, worst_grad

import torch
import torch.distributed as dist
import torch.nn.functional as F

from dstraining_b200.models.gpt import GPT
from dstraining_b200.parallel import comm, topology


def toy_split(rep, tp, device, sequence: bool):
    g = torch.Generator().manual_seed(SEED)
    shape = (2, 8, 6) if sequence else (4, 8)
    width = 12 if sequence else 16
    X = torch.randn(*shape, generator=g).to(device).requires_grad_(True)
    A = torch.randn(shape[-1], width, generator=g).to(device).requires_grad_(True)
    B = torch.randn(width, shape[-1], generator=g).to(device).requires_grad_(True)
    ref = F.gelu(X @ A) @ B
    ref.sum().backward()

    w = width // tp.world
    cols = slice(tp.rank * w, (tp.rank + 1) * w)
    Xp = X.detach().clone().requires_grad_(True)
    Ai = A.detach()[:, cols].clone().requires_grad_(True)
    Bi = B.detach()[cols, :].clone().requires_grad_(True)
    if sequence:
        xs = comm.scatter_along_seq(Xp, tp)
        out = comm.reduce_scatter_along_seq(F.gelu(comm.gather_along_seq(xs, tp) @ Ai) @ Bi, tp)
        t = shape[1] // tp.world
        want = ref[:, tp.rank * t : (tp.rank + 1) * t]
    else:
        out = comm.reduce_from_tp_region(F.gelu(comm.copy_to_tp_region(Xp, tp) @ Ai) @ Bi, tp)
        want = ref
    out.sum().backward()
    tag = "g/ḡ" if sequence else "f/f̄"
    rep.close(f"{tag} forward", max_diff(out, want))
    rep.close(f"{tag} grad X", max_diff(Xp.grad, X.grad))
    rep.close(f"{tag} grad A shard", max_diff(Ai.grad, A.grad[:, cols]))
    rep.close(f"{tag} grad B shard", max_diff(Bi.grad, B.grad[cols, :]))


def seq_sharding(rep, tp, model, cfg, device):
    shapes = []
    hooks = [b.ln_1.register_forward_hook(lambda m, a, o: shapes.append(tuple(a[0].shape))) for b in model.blocks]
    idx, tgt = batch(cfg, 4, SEED + 1, device)
    with torch.no_grad():
        model(idx, tgt)
    for h in hooks:
        h.remove()
    want = (4, cfg.block_size // tp.world, cfg.n_embd)
    rep.flag(f"LayerNorm inputs are {want} in all {len(shapes)} blocks", all(s == want for s in shapes))


def model_checks(rep, tp, model, ref, cfg, device):
    ref_p = dict(ref.named_parameters())
    worst = max(max_diff(p.data, shard_of(model, n, p, ref_p[n].data, tp)) for n, p in model.named_parameters())
    rep.close(f"init: all {len(ref_p)} params are slices of the full weights", worst, atol=0.0)

    idx, tgt = batch(cfg, 4, SEED + 1, device)
    if cfg.vocab_parallel_loss:
        with torch.no_grad():
            logits, _ = model(idx)
            logits_ref, _ = ref(idx)
        _, loss = model(idx, tgt)
        _, loss_ref = ref(idx, tgt)
    else:
        logits, loss = model(idx, tgt)
        logits_ref, loss_ref = ref(idx, tgt)
    rep.close("logits", max_diff(logits, logits_ref))
    rep.close("loss", max_diff(loss, loss_ref))
    if tp.enabled:
        parts = [torch.empty_like(logits) for _ in range(tp.world)]
        dist.all_gather(parts, logits.detach().contiguous(), group=tp.group)
        rep.close("cross-rank logit identity", max(max_diff(p, parts[0]) for p in parts), atol=0.0)
    loss.backward()
    model.finalize_grads()
    loss_ref.backward()
    name, worst = worst_grad(model, ref, tp)
    rep.close(f"all grads (worst {name})", worst)
    model.zero_grad(set_to_none=True)
    ref.zero_grad(set_to_none=True)


def training(rep, tp, model, ref, cfg, device, steps=10):
    idx, tgt = batch(cfg, 4, SEED + 2, device)
    opt = torch.optim.Adam(model.parameters(), lr=1e-3)
    opt_ref = torch.optim.Adam(ref.parameters(), lr=1e-3)
    losses, worst = [], 0.0
    for _ in range(steps):
        _, loss = model(idx, tgt)
        _, loss_ref = ref(idx, tgt)
        worst = max(worst, abs(loss.item() - loss_ref.item()))
        losses.append(loss.item())
        opt.zero_grad(set_to_none=True)
        opt_ref.zero_grad(set_to_none=True)
        loss.backward()
        model.finalize_grads()
        loss_ref.backward()
        opt.step()
        opt_ref.step()
    rep.close(f"{steps}-step Adam trajectory", worst, atol=1e-4)
    rep.flag(f"loss falls {losses[0]:.4f} -> {losses[-1]:.4f}", losses[-1] < losses[0])


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--sp", action="store_true")
    ap.add_argument("--recompute", action="store_true")
    ap.add_argument("--recompute-blocks", action="store_true", help="full activation recompute of every block")
    ap.add_argument("--vp", action="store_true")
    ap.add_argument("--device", default=None)
    a = ap.parse_args()
    device = start(a.device)
    tp = topology.make_tp_context()
    rep = Report()
    cfg = small_config(sequence_parallel=a.sp, vocab_parallel_loss=a.vp)
    rep.say(f"tp={tp.world} sp={a.sp} recompute={a.recompute} vp={a.vp}")
    toy_split(rep, tp, device, sequence=False)
    if a.sp:
        toy_split(rep, tp, device, sequence=True)
    model = GPT(replace(cfg, recompute_attention=a.recompute, recompute_blocks=a.recompute_blocks), tp,
                seed=SEED).to(device)
    ref = GPT(cfg, topology.SINGLE, seed=SEED).to(device)
    if a.sp and tp.enabled:
        seq_sharding(rep, tp, model, cfg, device)
    model_checks(rep, tp, model, ref, cfg, device)
    training(rep, tp, model, ref, cfg, device)
    rep.finish(device)


if __name__ == "__main__":
    main()
