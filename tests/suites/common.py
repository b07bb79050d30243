"""Shared helpers for the multi-rank correctness suites.

Every suite builds the parallel model AND a single-process model with the
same seed; decomposition-invariant init makes the latter hold exactly the
full tensors that the parallel model shards, so weights, logits, losses and
gradients can be compared slice by slice with no weight copying. The suites
run as N ranks (gloo on CPU, NCCL with ``--device cuda``) and agree on one
verdict with an all-reduce, exiting 0 on success.
"""

from __future__ import annotations

import os
import sys

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), "..", ".."))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from dstraining_b200.models.gpt import GPTConfig  # noqa: E402
from dstraining_b200.models.layers import ColumnParallelLinear, RowParallelLinear  # noqa: E402
from dstraining_b200.parallel import topology  # noqa: E402

SEED = 1234
ATOL = 1e-5


class Report:
    def __init__(self):
        self.ok = True

    def say(self, msg: str, only_rank0: bool = True) -> None:
        if not only_rank0 or dist.get_rank() == 0:
            print(msg, flush=True)

    def close(self, name: str, diff: float, atol: float = ATOL, only_rank0: bool = True) -> bool:
        good = diff <= atol
        self.ok &= good
        self.say(f"  [{'PASS' if good else 'FAIL'}] {name}: max abs diff {diff:.3e} (atol {atol:g})", only_rank0)
        return good

    def flag(self, name: str, good: bool, only_rank0: bool = True) -> bool:
        self.ok &= bool(good)
        self.say(f"  [{'PASS' if good else 'FAIL'}] {name}", only_rank0)
        return bool(good)

    def finish(self, device) -> None:
        verdict = torch.tensor(0 if self.ok else 1, device=device)
        dist.all_reduce(verdict)
        good = verdict.item() == 0
        self.say("\nALL PASS" if good else "\nFAILED")
        dist.destroy_process_group()
        sys.exit(0 if good else 1)


def start(device_arg):
    topology.init_distributed()
    if device_arg:
        device = torch.device(device_arg)
        if device.type == "cuda" and device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
    else:
        device = topology.default_device()
    torch.manual_seed(SEED)
    return device


def small_config(**kw) -> GPTConfig:
    base = dict(vocab_size=512, block_size=64, n_layer=4, n_head=8, n_embd=128, dropout=0.0)
    base.update(kw)
    return GPTConfig(**base)


# |g| at or below this fraction of the largest |g| of the same parameter and
# step is within a few hundred ulps of fp32 summation noise for these sizes.
NOISE_FLOOR = 1e-5


class NoiseLevelGrads:
    """Elements of a reference model whose gradient was, at some step, non-zero
    but at the rounding-noise level (``|g| <= NOISE_FLOOR * max |g|`` of the
    same parameter). Adam divides each update by the gradient's own running
    magnitude, so for these elements a different summation order - which may
    even flip the sign of such a gradient - moves them by up to lr per step in
    either run; comparisons hold them to that bound instead of the tight
    tolerance. Examples: the key part of the qkv bias, whose exact gradient is
    zero (softmax is unchanged when every key of a row shifts by the same
    q.b), and an embedding row whose token's contributions cancel."""

    def __init__(self):
        self.mask = {}

    def record(self, model: torch.nn.Module) -> None:
        """Call after each backward of the reference model."""
        for name, p in model.named_parameters():
            if p.grad is None:
                continue
            g = p.grad.detach()
            tiny = (g != 0) & (g.abs() <= NOISE_FLOOR * g.abs().max())
            self.mask[name] = self.mask[name] | tiny if name in self.mask else tiny

    def compare(self, pairs):
        """``pairs``: (reference parameter name, tensor, reference tensor).
        Returns (max |diff| over the other elements, max |diff| over the
        noise-level ones, number of noise-level elements)."""
        worst, worst_noisy, n_noisy = 0.0, 0.0, 0
        for name, x, r in pairs:
            diff = (x.float() - r.float()).abs()
            mask = self.mask.get(name)
            if mask is not None and mask.any():
                n_noisy += int(mask.sum())
                worst_noisy = max(worst_noisy, diff[mask].max().item())
                diff = diff[~mask]
            if diff.numel():
                worst = max(worst, diff.max().item())
        return worst, worst_noisy, n_noisy


def max_diff(a: torch.Tensor, b: torch.Tensor) -> float:
    return (a.float() - b.float()).abs().max().item()


def shard_of(model, name: str, local: torch.Tensor, full: torch.Tensor, tp) -> torch.Tensor:
    """The piece of a full-model tensor (weight or grad) that parameter
    ``name`` of a TP-sharded model holds."""
    if local.shape == full.shape:
        return full
    owner = model.get_submodule(name.rsplit(".", 1)[0])
    leaf = name.rsplit(".", 1)[1]
    if isinstance(owner, ColumnParallelLinear):
        n = local.shape[0]
        return full[tp.rank * n : (tp.rank + 1) * n]
    if isinstance(owner, RowParallelLinear) and leaf == "weight":
        n = local.shape[1]
        return full[:, tp.rank * n : (tp.rank + 1) * n]
    raise AssertionError(f"unexpected sharded parameter {name}")


def worst_grad(model, ref_model, tp, name_map=None):
    ref = dict(ref_model.named_parameters())
    name_map = name_map or (lambda n: n)
    worst_name, worst = None, -1.0
    for name, p in model.named_parameters():
        full = ref[name_map(name)].grad
        d = max_diff(p.grad, shard_of(model, name, p, full, tp))
        if d > worst:
            worst_name, worst = name, d
    return worst_name, worst


def batch(cfg: GPTConfig, n: int, seed: int, device):
    g = torch.Generator().manual_seed(seed)
    idx = torch.randint(0, cfg.vocab_size, (n, cfg.block_size), generator=g)
    tgt = torch.randint(0, cfg.vocab_size, (n, cfg.block_size), generator=g)
    return idx.to(device), tgt.to(device)
