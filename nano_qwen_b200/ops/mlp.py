"""SwiGLU on the packed gate|up GEMM output.

The dense FFN runs one GEMM against the contiguous [gate; up] weight
([2I, H]), so its output row is [g_0..g_{I-1}, u_0..u_{I-1}]; this kernel
writes ``silu(g) * u`` and its backward writes the packed [dg | du] gradient
that feeds the fused gate|up dgrad/wgrad GEMMs.  Replaces reference:
model/ffn.py:26 (three eager kernels) and kernels/swiglu.py:21-64.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from ._ext import ext
from .common import rows


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
