"""Python face of the tcgen05 GEMM (``csrc/gemm.cuh``).

``gemm(A, a_mn, B, b_mn, epi, ...)`` computes ``op(A) . op(B)^T`` where
``A`` is ``[M, K]`` (K-major) or, with ``a_mn``, ``[K, M]`` (M-major); ``B``
is ``[N, K]`` or, with ``b_mn``, ``[K, N]``. The three products a linear layer
needs:

    y  = x W^T      gemm(x,  False, W, False)
    dx = dy W       gemm(dy, False, W, True)
    dW = dy^T x     gemm(dy, True,  x, True)      (weight_grad: split-K)
"""

from __future__ import annotations

from typing import Optional

import torch

from . import native

EPI_STORE = 0
EPI_BIAS = 1
EPI_BIAS_GELU = 2
EPI_BIAS_RESID = 3
EPI_DGELU = 4


def gemm(
    a: torch.Tensor,
    a_mn: bool,
    b: torch.Tensor,
    b_mn: bool,
    epi: int = EPI_STORE,
    bias: Optional[torch.Tensor] = None,
    aux: Optional[torch.Tensor] = None,
    aux_out: Optional[torch.Tensor] = None,
    out: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    return native.lib().gemm(a, a_mn, b, b_mn, epi, bias, aux, aux_out, out)


def weight_grad(dy2: torch.Tensor, x2: torch.Tensor) -> torch.Tensor:
    """dW = dy^T x for dy [tokens, out], x [tokens, in] -> [out, in] (bf16),
    split over the token dimension with a fixed-order fp32 reduction."""
    return native.lib().gemm_splitk(dy2, True, x2, True, 0, None)


def bias_grad(dy2: torch.Tensor) -> torch.Tensor:
    return native.lib().colsum_bf16(dy2)
