"""Vision-tower ops: LayerNorm, GELU and patch embedding as a GEMM.

Patch embedding with kernel = stride = P is an im2col that is a pure
reshape/permute of the image ([B, C, H, W] -> [B, (H/P)(W/P), C*P*P]) followed
by one GEMM against the conv weight viewed as [D, C*P*P]; on GPU the K
dimension is zero-padded to a multiple of 8 so TMA row strides are 16-byte
multiples.  Replaces reference: model/vision/patch_embed.py:13-34 (Conv2d),
model/vision/vit.py:20-61 (nn.LayerNorm, nn.GELU).
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn.functional as F

from ._ext import ext
from .common import grad_buffer, rows
from .linear import linear


class _LayerNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, eps, out_dtype):
        shape = x.shape
        y, mean, rstd = ext().layernorm_fwd(rows(x), weight, bias, float(eps), out_dtype)
        ctx.save_for_backward(rows(x), weight, mean, rstd)
        ctx.has_bias = bias is not None
        ctx.bias = bias
        return y.view(shape)

    @staticmethod
    def backward(ctx, dy):
        x, weight, mean, rstd = ctx.saved_tensors
        dw = grad_buffer(weight) if weight.requires_grad else None
        b = ctx.bias
        db = grad_buffer(b) if (b is not None and b.requires_grad) else None
        dx = ext().layernorm_bwd(rows(dy), x, weight, mean, rstd, dw, db)
        return dx.view(dy.shape).to(x.dtype), None, None, None, None


def layer_norm(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor], eps: float,
               out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    if x.is_cuda:
        return _LayerNormFn.apply(x, weight, bias, eps, out_dtype or x.dtype)
    return F.layer_norm(x, (x.shape[-1],), weight, bias, eps)


class _GeluFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        ctx.save_for_backward(x)
        return ext().gelu_fwd(x.contiguous())

    @staticmethod
    def backward(ctx, dy):
        (x,) = ctx.saved_tensors
        return ext().gelu_bwd(dy.contiguous(), x)


def gelu(x: torch.Tensor) -> torch.Tensor:
    """Exact (erf) GELU, as ``nn.GELU()``."""
    if x.is_cuda:
        return _GeluFn.apply(x)
    return F.gelu(x)


def patchify(pixel_values: torch.Tensor, patch: int) -> torch.Tensor:
    """[B, C, H, W] -> [B, (H/P)*(W/P), C*P*P] in conv-weight (C, kh, kw) order."""
    B, C, H, W = pixel_values.shape
    x = pixel_values.reshape(B, C, H // patch, patch, W // patch, patch)
    x = x.permute(0, 2, 4, 1, 3, 5)
    return x.reshape(B, (H // patch) * (W // patch), C * patch * patch)
