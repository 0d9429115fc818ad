"""Qwen3-VL: ViT -> DeepStack -> Merger -> Qwen3 language model.

Same modules, parameter names and forward signature as the reference's
``Qwen3VLModel`` (vision_encoder, deepstack, merger, language_model;
``forward(input_ids, pixel_values, image_token_mask, position_ids,
attention_mask, labels)``; reference: model/multimodal.py:22-143).
Differences: visual tokens are scattered into the text embeddings with one
masked scatter (the reference looped per token in Python), the loss is the
fused lm_head + CE, and multimodal RoPE is actually applied: when
``image_grid_thw`` (or the merged image grids) are known, per-token
(t, h, w) positions rotate the q/k heads through the fused RoPE kernel.
"""

from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn as nn

from .. import ops
from ..config import ModelConfig
from .transformer import Qwen3Model, key_range_mask, shift_targets
from .vision.deepstack import DeepStack
from .vision.merger import VisionMerger
from .vision.mrope import build_mrope_position_ids, mrope_tables
from .vision.vit import VisionTransformer


class Qwen3VLModel(nn.Module):
    def __init__(self, config: ModelConfig):
        super().__init__()
        assert config.vision_enabled, "vision_enabled must be True for Qwen3VLModel"
        self.config = config
        self.vision_encoder = VisionTransformer(config)
        self.deepstack = DeepStack(config.vision_hidden_size, config.hidden_size,
                                   len(config.vision_deepstack_layers) + 1)
        self.merger = VisionMerger(config.hidden_size, config.hidden_size,
                                   config.vision_merger_spatial_factor)
        self.language_model = Qwen3Model(config)
        scaling = config.rope_scaling or {}
        self.mrope_section = scaling.get("mrope_section") if scaling.get("type") == "mrope" else None
        self.use_mrope = True

    def encode_images(self, pixel_values: torch.Tensor) -> torch.Tensor:
        vit = self.vision_encoder(pixel_values)
        fused = self.deepstack(vit["intermediate_states"], vit["last_hidden_state"])
        g = int(math.isqrt(fused.shape[1]))
        return self.merger(fused, g, g)

    def forward(self, input_ids: torch.Tensor, pixel_values: Optional[torch.Tensor] = None,
                image_token_mask: Optional[torch.Tensor] = None,
                position_ids: Optional[torch.Tensor] = None,
                attention_mask: Optional[torch.Tensor] = None,
                labels: Optional[torch.Tensor] = None,
                image_grid_thw: Optional[torch.Tensor] = None,
                return_logits: Optional[bool] = None) -> dict:
        lm = self.language_model
        h = lm.embed(input_ids)
        rope = None
        if pixel_values is not None and image_token_mask is not None:
            vis = self.encode_images(pixel_values)                 # [n_img, m, H]
            flat = vis.reshape(-1, vis.shape[-1]).to(h.dtype)
            mask = image_token_mask.bool()
            n = min(int(mask.sum()), flat.shape[0])
            if n > 0:
                idx = mask.reshape(-1).nonzero(as_tuple=True)[0][:n]
                h = h.reshape(-1, h.shape[-1]).index_copy(0, idx, flat[:n]).view_as(h)
            if self.use_mrope:
                B, S = input_ids.shape
                if image_grid_thw is None:
                    g = int(math.isqrt(vis.shape[1]))
                    image_grid_thw = torch.tensor([[1, g, g]] * vis.shape[0])
                base = position_ids if position_ids is not None else \
                    torch.arange(S, device=input_ids.device).unsqueeze(0).expand(B, S)
                pos = build_mrope_position_ids(base, image_grid_thw, mask)
                rope = mrope_tables(self.config.head_dim, self.config.rope_theta, pos,
                                    self.mrope_section)
        x, aux_total, n_moe = lm.hidden(input_ids, position_ids, key_range_mask(attention_mask), None,
                                        inputs_embeds=h, rope=rope)
        if return_logits is None:
            return_logits = labels is None
        logits = ops.linear(x, lm.lm_head_ref(x.dtype)) if return_logits else None
        loss = None
        if labels is not None:
            loss = ops.linear_cross_entropy(x, lm.lm_head_ref(x.dtype), shift_targets(labels))
            if n_moe > 0:
                loss = loss + self.config.router_aux_loss_coef * (aux_total / n_moe)
        return {"logits": logits, "loss": loss, "aux_loss": aux_total if n_moe else None,
                "hidden_states": x}
