"""Parameter-holding building blocks shared by the language and vision models.

Modules here own parameters under the reference's names; their forward passes
call ``nano_qwen_b200.ops`` (sm_100a kernels on CUDA tensors, plain PyTorch on
CPU tensors).
"""

from __future__ import annotations

from typing import Optional, Sequence

import torch
import torch.nn as nn

from .. import ops


class Linear(nn.Module):
    """``y = x W^T (+ b)``; the weight layout of ``nn.Linear``."""

    def __init__(self, in_features: int, out_features: int, bias: bool = False):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.weight = nn.Parameter(torch.empty(out_features, in_features))
        self.bias = nn.Parameter(torch.zeros(out_features)) if bias else None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return fused_linear(x, [self], compute_dtype_of(x))


def compute_dtype_of(x: torch.Tensor) -> torch.dtype:
    """GEMM input dtype: bf16 on the GPU (the tcgen05 kernels' operand type,
    whatever the activation's dtype, e.g. an fp32 residual stream), the
    input's own dtype on the CPU."""
    return torch.bfloat16 if x.is_cuda else x.dtype


def fused_linear(x: torch.Tensor, linears: Sequence[Linear], dtype: torch.dtype) -> torch.Tensor:
    """One GEMM over the concatenated weights of ``linears`` (rows stacked).

    Tensor-parallel layers (``tp_mode`` set by ``parallel.tensor_parallel``)
    gather their input (column-parallel) or reduce their output (row-parallel).
    """
    wref = ops.weight_ref([l.weight for l in linears], dtype)
    bias = None
    if linears[0].bias is not None:
        bias = torch.cat([l.bias for l in linears]) if len(linears) > 1 else linears[0].bias
    if x.dtype != dtype:
        x = x.to(dtype)
    mode = getattr(linears[0], "tp_mode", None)
    if mode is None:
        return ops.linear(x, wref, bias)
    from ..parallel.tensor_parallel import tp_input, tp_output
    if mode == "col":
        return ops.linear(tp_input(x, linears[0]), wref, bias)
    y = tp_output(ops.linear(x, wref), linears[0])
    return y + bias.to(y.dtype) if bias is not None else y


class RMSNorm(nn.Module):
    """RMSNorm with a learnable scale (reference: model/norm.py:11-22)."""

    def __init__(self, hidden_size: int, eps: float = 1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden_size))
        self.eps = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return ops.rms_norm(x, self.weight, self.eps)


class LayerNorm(nn.Module):
    """LayerNorm with the ``nn.LayerNorm`` parameter names (weight, bias)."""

    def __init__(self, hidden_size: int, eps: float = 1e-5):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden_size))
        self.bias = nn.Parameter(torch.zeros(hidden_size))
        self.eps = eps
        self.normalized_shape = (hidden_size,)

    def forward(self, x: torch.Tensor, out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
        return ops.layer_norm(x, self.weight, self.bias, self.eps, out_dtype)
