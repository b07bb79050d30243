"""bf16 parameters with fp32 master weights and Adam.

Model parameters, activations and gradients are bf16; the authoritative
weights and the Adam moments are fp32. Each step upcasts the gradient,
updates the fp32 master with Adam and rounds the master once into the bf16
parameter (so ``param == master.to(bf16)`` bitwise after every step). bf16
has fp32's exponent range, so no loss scaling is needed. Same contract as the
reference's ``dst/precision.py:27-44``: ``model_params``, ``master_params``
and an ``inner`` ``torch.optim.Adam`` whose ``state[master]`` holds
``exp_avg``/``exp_avg_sq``/``step``.

On CUDA the whole update - upcast, both moment updates, bias correction,
the master update and the bf16 write-back - is one native multi-tensor
kernel launch per step over every parameter (the reference runs
``torch.optim.Adam`` plus a Python loop of casts and copies). The kernel
implements the same update as ``torch.optim.Adam`` (Kingma & Ba, Algorithm
1 with ``eps`` added after the bias-corrected square root) and writes
straight into ``inner.state``, so the two paths are interchangeable. The
kernel also applies decoupled weight decay (``weight_decay`` with
``decoupled_weight_decay=True``, i.e. AdamW); Adam options it does not
implement (coupled ``weight_decay``, ``amsgrad``, ``maximize``) take the
PyTorch path of the same step, as in the reference.
"""

from __future__ import annotations

from typing import Iterable, List

import torch

from ..ops import native


class MasterWeightOptimizer:
    """bf16 model parameters with fp32 master copies and an inner ``torch.optim.Adam``
    over the masters (``dst/precision.py:27-44``): ``step()`` upcasts the gradients,
    updates the masters and copies them back to the bf16 parameters. On CUDA bf16
    the whole update is one multi-tensor native kernel; ``model_params``,
    ``master_params`` and ``inner.state`` stay available."""

    def __init__(self, params: Iterable[torch.nn.Parameter], **adam_kwargs):
        self.model_params: List[torch.nn.Parameter] = [p for p in params if p.requires_grad]
        self.master_params = [p.detach().clone().float().requires_grad_(False) for p in self.model_params]
        self.inner = torch.optim.Adam(self.master_params, **adam_kwargs)
        self._native = native.enabled() and all(
            p.is_cuda and p.dtype == torch.bfloat16 for p in self.model_params
        )
        self._tables = None

    def zero_grad(self, set_to_none: bool = True) -> None:
        """Clear the bf16 parameters' gradients (and the masters')."""
        for p in self.model_params:
            if set_to_none:
                p.grad = None
            elif p.grad is not None:
                p.grad.zero_()

    def _state(self, master: torch.Tensor):
        st = self.inner.state[master]
        if not st:
            st["step"] = torch.zeros((), dtype=torch.float32)
            st["exp_avg"] = torch.zeros_like(master, memory_format=torch.preserve_format)
            st["exp_avg_sq"] = torch.zeros_like(master, memory_format=torch.preserve_format)
        return st

    def _native_supports(self) -> bool:
        group = self.inner.param_groups[0]
        coupled_decay = group.get("weight_decay", 0.0) and not group.get("decoupled_weight_decay", False)
        return not (group.get("amsgrad") or group.get("maximize") or coupled_decay)

    def step(self) -> None:
        """One Adam step on the fp32 masters, then bf16 parameters = masters."""
        if self._native and self._native_supports():
            self._native_step()
            return
        for mp, master in zip(self.model_params, self.master_params):
            master.grad = None if mp.grad is None else mp.grad.float()
        self.inner.step()
        for mp, master in zip(self.model_params, self.master_params):
            mp.data.copy_(master)

    def _native_step(self) -> None:
        group = self.inner.param_groups[0]
        lr = float(group["lr"])
        beta1, beta2 = group["betas"]
        eps = float(group["eps"])
        live = [i for i, p in enumerate(self.model_params) if p.grad is not None]
        if not live:
            return
        params, grads, masters, m1, m2 = [], [], [], [], []
        step = None
        for i in live:
            master = self.master_params[i]
            st = self._state(master)
            st["step"] += 1
            step = float(st["step"])
            params.append(self.model_params[i].data)
            grads.append(self.model_params[i].grad)
            masters.append(master)
            m1.append(st["exp_avg"])
            m2.append(st["exp_avg_sq"])
        native.lib().adam_master_step(params, grads, masters, m1, m2, lr, beta1, beta2, eps, step,
                                      weight_decay=float(group.get("weight_decay", 0.0)))
