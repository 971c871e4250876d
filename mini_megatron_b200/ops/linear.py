"""GEMM helpers for linear layers on the native path.

Weights are ``[out, in]`` (row-major, like ``nn.Linear``) in bf16; activations
are row-major ``[tokens, features]``.  Every helper maps to ONE launch of the
tcgen05 GEMM with the matching operand majors and epilogue:

=============  ==========================  ======================
helper         math                        operands (A, B)
=============  ==========================  ======================
linear_fwd     y  = x W^T                  x K-major, W K-major
linear_dgrad   dx = dy W                   dy K-major, W MN-major
linear_wgrad   dW += dy^T x (fp32 accum)   dy MN-major, x MN-major
=============  ==========================  ======================
"""
from __future__ import annotations

import torch

from . import native

EPI_BF16, EPI_F32, EPI_F32_ACC, EPI_GELU, EPI_RESID, EPI_DGELU = range(6)


def linear_fwd(x2d, w, out=None, epi=EPI_BF16, aux=None, resid=None, alpha=1.0):
    C = native()
    M, N = x2d.shape[0], w.shape[0]
    if out is None:
        dtype = torch.bfloat16 if epi in (EPI_BF16, EPI_GELU, EPI_DGELU) else torch.float32
        out = torch.empty(M, N, device=x2d.device, dtype=dtype)
    C.gemm(x2d, False, w, False, out, epi, aux=aux, resid=resid, alpha=alpha)
    return out


def linear_gelu_fwd(x2d, w):
    """(gelu(h), gelu'(h)) with h = x W^T, both bf16 -- fc1 with the GELU fused in the epilogue.

    The derivative is saved instead of h: the backward's fc2 dgrad epilogue then
    only multiplies by it (EPI_DGELU)."""
    grad = torch.empty(x2d.shape[0], w.shape[0], device=x2d.device, dtype=torch.bfloat16)
    act = torch.empty_like(grad)
    native().gemm(x2d, False, w, False, act, EPI_GELU, aux=grad)
    return act, grad


def linear_dgrad(dy2d, w, out=None, epi=EPI_BF16, aux=None):
    C = native()
    M, N = dy2d.shape[0], w.shape[1]
    if out is None:
        dtype = torch.bfloat16 if epi in (EPI_BF16, EPI_GELU, EPI_DGELU) else torch.float32
        out = torch.empty(M, N, device=dy2d.device, dtype=dtype)
    C.gemm(dy2d, False, w, True, out, epi, aux=aux)
    return out


def linear_wgrad(dy2d, x2d, dw_fp32):
    """dW(fp32) += dy^T x ; split-K with atomics when the output is small."""
    native().gemm(dy2d, True, x2d, True, dw_fp32, EPI_F32_ACC)
    return dw_fp32
