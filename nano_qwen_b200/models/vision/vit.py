"""Vision transformer encoder (reference: model/vision/vit.py:20-141).

Same parameter names (patch_embed, pos_embed, blocks.{i}.{norm1,attn.qkv,
attn.proj,norm2,mlp.fc1,mlp.fc2}, norm) and behaviour: pre-LN blocks with
non-causal multi-head attention and an exact-GELU MLP, learned position
embeddings bilinearly interpolated for other resolutions, intermediate
states collected at ``vision_deepstack_layers``.  Execution: LayerNorm, GELU
and attention are the sm_100a kernels (the attention kernel in non-causal
mode, head_dim 64), projections are tcgen05 GEMMs.
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from ... import ops
from ...config import ModelConfig
from ..layers import LayerNorm, Linear
from .patch_embed import PatchEmbedding


def _dt(x):
    return torch.bfloat16 if x.is_cuda else x.dtype


class ViTMLP(nn.Module):
    def __init__(self, hidden_size: int, intermediate_size: int):
        super().__init__()
        self.fc1 = Linear(hidden_size, intermediate_size, bias=True)
        self.fc2 = Linear(intermediate_size, hidden_size, bias=True)

    def forward(self, x):
        return self.fc2(ops.gelu(self.fc1(x)))


class ViTAttention(nn.Module):
    def __init__(self, hidden_size: int, num_heads: int):
        super().__init__()
        self.num_heads = num_heads
        self.head_dim = hidden_size // num_heads
        self.qkv = Linear(hidden_size, 3 * hidden_size, bias=True)
        self.proj = Linear(hidden_size, hidden_size, bias=True)

    def forward(self, x):
        B, N, D = x.shape
        qkv = self.qkv(x).view(B, N, 3, self.num_heads, self.head_dim)
        q, k, v = qkv.unbind(2)
        o = ops.full_attention(q, k, v, causal=False)
        return self.proj(o.reshape(B, N, D))


class ViTBlock(nn.Module):
    def __init__(self, hidden_size: int, num_heads: int, intermediate_size: int):
        super().__init__()
        self.norm1 = LayerNorm(hidden_size, eps=1e-5)
        self.attn = ViTAttention(hidden_size, num_heads)
        self.norm2 = LayerNorm(hidden_size, eps=1e-5)
        self.mlp = ViTMLP(hidden_size, intermediate_size)

    def forward(self, x):
        dt = _dt(x)
        x = x + self.attn(self.norm1(x, dt)).to(x.dtype)
        x = x + self.mlp(self.norm2(x, dt)).to(x.dtype)
        return x


class VisionTransformer(nn.Module):
    def __init__(self, config: ModelConfig):
        super().__init__()
        self.config = config
        self.patch_embed = PatchEmbedding(config)
        self.pos_embed = nn.Parameter(torch.zeros(1, config.vision_num_patches, config.vision_hidden_size))
        self.blocks = nn.ModuleList([ViTBlock(config.vision_hidden_size, config.vision_num_attention_heads,
                                              config.vision_intermediate_size)
                                     for _ in range(config.vision_num_hidden_layers)])
        self.norm = LayerNorm(config.vision_hidden_size, eps=1e-5)
        self.deepstack_layers = set(config.vision_deepstack_layers or [])
        nn.init.trunc_normal_(self.pos_embed, std=0.02)
        for m in self.modules():
            if isinstance(m, Linear):
                nn.init.normal_(m.weight, std=0.02)

    def forward(self, pixel_values: torch.Tensor) -> dict:
        x = self.patch_embed(pixel_values).float()      # residual stream in fp32
        pos = self.pos_embed if x.shape[1] == self.pos_embed.shape[1] else self._interpolate_pos_embed(x)
        x = x + pos
        inter = []
        for i, blk in enumerate(self.blocks):
            x = blk(x)
            if i in self.deepstack_layers:
                inter.append(x)
        x = self.norm(x, torch.float32)
        return {"last_hidden_state": x, "intermediate_states": inter}

    def _interpolate_pos_embed(self, x):
        n_new, n_old, dim = x.shape[1], self.pos_embed.shape[1], x.shape[-1]
        h0 = int(math.sqrt(n_old))
        h1 = int(math.sqrt(n_new))
        p = self.pos_embed.reshape(1, h0, h0, dim).permute(0, 3, 1, 2)
        p = F.interpolate(p, size=(h1, h1), mode="bilinear", align_corners=False)
        return p.permute(0, 2, 3, 1).reshape(1, -1, dim)
