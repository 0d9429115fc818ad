"""Vision-language merger: f x f spatial patch merge, then LayerNorm -> Linear
-> GELU -> Linear (reference: model/vision/merger.py:15-57; parameter names
mlp.0 / mlp.1 / mlp.3 as in the reference's ``nn.Sequential``)."""

from __future__ import annotations

import torch
import torch.nn as nn

from ... import ops
from ..layers import LayerNorm, Linear


class GELU(nn.Module):
    def forward(self, x):
        return ops.gelu(x)


class VisionMerger(nn.Module):
    def __init__(self, vision_hidden_size: int, llm_hidden_size: int, spatial_factor: int = 2):
        super().__init__()
        self.spatial_factor = spatial_factor
        merged = vision_hidden_size * spatial_factor ** 2
        self.mlp = nn.Sequential(LayerNorm(merged, eps=1e-5), Linear(merged, llm_hidden_size, bias=True),
                                 GELU(), Linear(llm_hidden_size, llm_hidden_size, bias=True))
        for m in self.mlp:
            if isinstance(m, Linear):
                nn.init.normal_(m.weight, std=0.02)

    def forward(self, visual_tokens: torch.Tensor, grid_h: int, grid_w: int) -> torch.Tensor:
        B, N, D = visual_tokens.shape
        f = self.spatial_factor
        assert grid_h % f == 0 and grid_w % f == 0, "grid not divisible by spatial_factor"
        x = visual_tokens.view(B, grid_h // f, f, grid_w // f, f, D).permute(0, 1, 3, 2, 4, 5)
        x = x.reshape(B, (grid_h // f) * (grid_w // f), f * f * D)
        dt = torch.bfloat16 if x.is_cuda else x.dtype
        h = self.mlp[0](x, dt)
        h = self.mlp[1](h)
        h = self.mlp[2](h)
        return self.mlp[3](h)
