"""SwiGLU on the packed gate|up GEMM output.

The dense FFN runs one GEMM against the contiguous [gate; up] weight
([2I, H]), so its output row is [g_0..g_{I-1}, u_0..u_{I-1}]; this kernel
writes ``silu(g) * u`` and its backward writes the packed [dg | du] gradient
that feeds the fused gate|up dgrad/wgrad GEMMs.  ``linear_swiglu`` goes one
step further on CUDA: the gate|up GEMM's epilogue applies the gating itself
(``gemm_nt_swiglu``), so ``h`` never takes a separate pass over ``gu``.
Replaces reference: model/ffn.py:26 (three eager kernels) and
kernels/swiglu.py:21-64.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from ._ext import ext
from .common import rows
from .linear import WeightRef, linear_backward


class _SwiGLUFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gu):
        shape = gu.shape
        g2 = rows(gu)
        h = ext().swiglu_fwd(g2)
        ctx.save_for_backward(g2)
        ctx.shape = shape
        return h.view(*shape[:-1], shape[-1] // 2)

    @staticmethod
    def backward(ctx, dh):
        (g2,) = ctx.saved_tensors
        dgu = ext().swiglu_bwd(rows(dh), g2)
        return dgu.view(ctx.shape)


def swiglu_packed(gu: torch.Tensor) -> torch.Tensor:
    """gu [..., 2I] -> silu(gu[..., :I]) * gu[..., I:]."""
    if gu.is_cuda:
        return _SwiGLUFn.apply(gu)
    g, u = gu.chunk(2, dim=-1)
    return F.silu(g) * u


class _LinearSwiGLUFn(torch.autograd.Function):
    """h = silu(x Wg^T) * (x Wu^T) with W = [Wg; Wu] one fused weight."""

    @staticmethod
    def forward(ctx, x, wref: WeightRef, *anchors):
        x2 = rows(x)
        gu, h = ext().gemm_nt_swiglu(x2, wref.compute)
        ctx.save_for_backward(x2, gu)
        ctx.wref = wref
        ctx.in_shape = x.shape
        return h.view(*x.shape[:-1], h.shape[-1])

    @staticmethod
    def backward(ctx, dh):
        x2, gu = ctx.saved_tensors
        dgu = ext().swiglu_bwd(rows(dh), gu)
        dx = linear_backward(dgu, x2, ctx.wref, ctx.needs_input_grad[0], ctx.in_shape)
        return (dx, None) + (None,) * len(ctx.wref.anchors)


def linear_swiglu_supported(x: torch.Tensor, wref: WeightRef) -> bool:
    return x.is_cuda and x.dtype == torch.bfloat16 and wref.compute.dtype == torch.bfloat16 \
        and wref.compute.dim() == 2 and wref.compute.shape[0] % 256 == 0 \
        and wref.compute.is_contiguous() and x.shape[-1] % 8 == 0


def linear_swiglu(x: torch.Tensor, wref: WeightRef) -> torch.Tensor:
    """silu(g) * u for [g | u] = x W^T, W = [gate; up] ([2I, H], I % 128 == 0)."""
    if torch.is_grad_enabled() and (x.requires_grad or wref.requires_grad):
        return _LinearSwiGLUFn.apply(x, wref, *wref.anchors)
    h = ext().gemm_nt_swiglu(rows(x), wref.compute)[1]
    return h.view(*x.shape[:-1], h.shape[-1])
