"""Patch embedding as im2col + one GEMM.

Keeps the reference's ``Conv2d`` parameter (``proj.weight`` [D, C, P, P] and
``proj.bias``; reference: model/vision/patch_embed.py:13-34) so checkpoints
load, but computes it as a reshape of the image into [B, N, C*P*P] rows and a
tcgen05 GEMM against the weight viewed as [D, C*P*P] (K zero-padded to a
multiple of 8 on GPU for 16-byte TMA strides).
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from ... import ops
from ...config import ModelConfig


class PatchEmbedding(nn.Module):
    def __init__(self, config: ModelConfig):
        super().__init__()
        self.patch_size = config.vision_patch_size
        self.proj = nn.Conv2d(config.vision_num_channels, config.vision_hidden_size,
                              kernel_size=config.vision_patch_size,
                              stride=config.vision_patch_size, bias=True)

    def forward(self, pixel_values: torch.Tensor) -> torch.Tensor:
        x = ops.patchify(pixel_values, self.patch_size)          # [B, N, C*P*P]
        w = self.proj.weight.reshape(self.proj.weight.shape[0], -1)
        if x.is_cuda:
            K = x.shape[-1]
            pad = (8 - K % 8) % 8
            xb = F.pad(x, (0, pad)).to(torch.bfloat16)
            wb = F.pad(w, (0, pad)).to(torch.bfloat16)
            y = ops.dense(xb, wb)
        else:
            y = x @ w.t()
        return y + self.proj.bias.to(y.dtype)
