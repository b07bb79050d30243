"""Selective activation recompute.

``recompute(fn, *args)`` runs ``fn`` without building a graph in forward and
keeps only its inputs; backward re-runs ``fn`` with grad enabled and
back-propagates through the fresh graph. The region must be deterministic and
RNG-free. Behaviour of the reference's ``dst/recompute.py:22-44``; the
autograd Function is named ``_Recompute`` because callers (and the reference's
test, ``tests/test_recompute.py:56-64``) patch ``_Recompute.forward`` to count
region entries.

On the native path the attention kernel is a flash kernel that never stores
the s x s probabilities, so there is nothing for recompute to discard there;
the flag only changes the PyTorch (oracle) path, where the attention matrix
is materialised on purpose.
"""

from __future__ import annotations

import torch


class _Recompute(torch.autograd.Function):
    @staticmethod
    def forward(ctx, fn, *args):
        ctx.fn = fn
        ctx.save_for_backward(*args)
        with torch.no_grad():
            return fn(*args)

    @staticmethod
    def backward(ctx, grad_out):
        inputs = [t.detach().requires_grad_(t.requires_grad) for t in ctx.saved_tensors]
        with torch.enable_grad():
            out = ctx.fn(*inputs)
        torch.autograd.backward(out, grad_out)
        return (None, *(t.grad for t in inputs))


def recompute(fn, *args) -> torch.Tensor:
    return _Recompute.apply(fn, *args)
