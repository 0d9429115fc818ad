"""Fused residual-add + RMSNorm.

The transformer's residual stream is kept in fp32 (as the reference's is under
autocast: the fp32 embedding output plus bf16 branch outputs promotes to fp32,
reference: model/transformer.py:60-72).  One kernel reads the fp32 stream and
the bf16 branch output, writes the updated fp32 stream and the bf16 normalised
activations for the next GEMM; the backward kernel fuses the RMSNorm gradient,
the residual gradient add, the weight-gradient reduction and the bf16 cast of
the branch gradient.  Replaces the eager composite of model/norm.py:17-22
(about five kernels per call) and reference kernels/rmsnorm.py:22-68.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import reference as ref
from ._ext import ext
from .common import grad_buffer, rows


class _AddRMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, resid, delta, weight, eps):
        shape = resid.shape
        r2 = rows(resid)
        d2 = rows(delta) if delta is not None else None
        h, y, rstd = ext().add_rmsnorm_fwd(r2, d2, weight, float(eps))
        ctx.save_for_backward(h, weight, rstd)
        ctx.has_delta = delta is not None
        ctx.shape = shape
        return h.view(shape), y.view(shape)

    @staticmethod
    def backward(ctx, dh, dy):
        h, weight, rstd = ctx.saved_tensors
        dw = grad_buffer(weight) if weight.requires_grad else None
        dh2 = rows(dh) if dh is not None else None
        dx, dx_bf16 = ext().add_rmsnorm_bwd(rows(dy), dh2, h, weight, rstd, dw)
        dx = dx.view(ctx.shape)
        ddelta = dx_bf16.view(ctx.shape) if ctx.has_delta else None
        return dx, ddelta, None, None


def add_rms_norm(resid: torch.Tensor, delta: Optional[torch.Tensor], weight: torch.Tensor,
                 eps: float) -> Tuple[torch.Tensor, torch.Tensor]:
    """h = resid + delta (fp32 stream); y = RMSNorm(h) * weight (compute dtype).

    Returns (h, y).  On CPU the math is plain PyTorch in the input dtype.
    """
    if resid.is_cuda:
        return _AddRMSNormFn.apply(resid, delta, weight, eps)
    h = resid if delta is None else resid + delta.to(resid.dtype)
    return h, ref.rms_norm(h, weight, eps)


class _RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, eps, out_dtype):
        shape = x.shape
        y, rstd = ext().rmsnorm_fwd(rows(x), weight, float(eps), out_dtype)
        ctx.save_for_backward(x, weight, rstd)
        return y.view(shape)

    @staticmethod
    def backward(ctx, dy):
        x, weight, rstd = ctx.saved_tensors
        dw = grad_buffer(weight) if weight.requires_grad else None
        dx = ext().rmsnorm_bwd(rows(dy), rows(x), weight, rstd, dw)
        return dx.view(x.shape).to(x.dtype), None, None, None


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float,
             out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    if x.is_cuda:
        return _RMSNormFn.apply(x, weight, eps, out_dtype or x.dtype)
    return ref.rms_norm(x, weight, eps)
