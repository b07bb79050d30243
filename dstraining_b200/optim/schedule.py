"""Learning-rate schedules: linear warm-up, then constant or cosine decay.

``lr_at(step, ...)`` is a pure function of the step, so a resumed run
continues the schedule exactly; ``set_lr(opt, lr)`` applies it to any of the
optimizers here (``torch.optim`` ones, ``MasterWeightOptimizer`` through its
inner Adam, ``FusedDPAdam`` whose bucket kernels read ``opt.lr`` when they
launch - so the rate must be set before the step's backward starts). The
reference trains at a constant rate (``train.py:98-101``).
"""

from __future__ import annotations

import math


def lr_at(step: int, base_lr: float, total_steps: int, warmup_steps: int = 0, schedule: str = "constant",
          min_lr: float = 0.0) -> float:
    """Rate for optimizer step ``step`` (0-based)."""
    if warmup_steps > 0 and step < warmup_steps:
        return base_lr * (step + 1) / warmup_steps
    if schedule == "constant":
        return base_lr
    if schedule == "cosine":
        span = max(1, total_steps - warmup_steps)
        t = min(1.0, max(0.0, (step - warmup_steps) / span))
        return min_lr + 0.5 * (base_lr - min_lr) * (1.0 + math.cos(math.pi * t))
    raise ValueError(f"unknown schedule {schedule!r}")


def set_lr(opt, lr: float) -> None:
    """Set the learning rate of any optimizer of this package (or a torch one)."""
    if hasattr(opt, "inner"):  # MasterWeightOptimizer
        opt = opt.inner
    if hasattr(opt, "param_groups"):
        for g in opt.param_groups:
            g["lr"] = lr
    else:  # FusedDPAdam
        opt.lr = lr
