"""SwiGLU feed-forward network (reference: model/ffn.py:16-34).

The gate and up weights are one contiguous [2I, H] fusion group: one GEMM
produces [g | u] and, on CUDA, applies the SiLU gating in its epilogue; one
GEMM projects down.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from .. import ops
from ..config import ModelConfig
from .layers import Linear, fused_linear


class SwiGLU(nn.Module):
    def __init__(self, hidden_size: int, intermediate_size: int, bias: bool = False):
        super().__init__()
        self.gate_proj = Linear(hidden_size, intermediate_size, bias)
        self.up_proj = Linear(hidden_size, intermediate_size, bias)
        self.down_proj = Linear(intermediate_size, hidden_size, bias)

    def fusion_groups(self):
        return [["gate_proj.weight", "up_proj.weight"]]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.is_cuda and getattr(self.gate_proj, "tp_mode", None) is None and self.gate_proj.bias is None:
            wref = ops.weight_ref([self.gate_proj.weight, self.up_proj.weight], x.dtype)
            if ops.linear_swiglu_supported(x, wref):
                h = ops.linear_swiglu(x, wref)
                return fused_linear(h, [self.down_proj], x.dtype)
        gu = fused_linear(x, [self.gate_proj, self.up_proj], x.dtype)
        h = ops.swiglu_packed(gu)
        return fused_linear(h, [self.down_proj], x.dtype)


def build_ffn(config: ModelConfig) -> SwiGLU:
    return SwiGLU(config.hidden_size, config.intermediate_size, bias=False)
