"""DeepStack: softmax-weighted fusion of per-level projections of ViT states
(reference: model/vision/deepstack.py:16-63; same parameters level_projs,
fusion_weights, norm and the same last-level fallback when the level count
does not match)."""

from __future__ import annotations

from typing import List

import torch
import torch.nn as nn

from ..layers import LayerNorm, Linear


class DeepStack(nn.Module):
    def __init__(self, vision_hidden_size: int, llm_hidden_size: int, num_levels: int):
        super().__init__()
        self.num_levels = num_levels
        self.level_projs = nn.ModuleList([Linear(vision_hidden_size, llm_hidden_size, bias=True)
                                          for _ in range(num_levels)])
        for p in self.level_projs:
            nn.init.normal_(p.weight, std=0.02)
        self.fusion_weights = nn.Parameter(torch.ones(num_levels))
        self.norm = LayerNorm(llm_hidden_size, eps=1e-5)

    def forward(self, intermediate_states: List[torch.Tensor], last_hidden_state: torch.Tensor):
        states = list(intermediate_states) + [last_hidden_state]
        if len(states) != self.num_levels:
            return self.norm(self.level_projs[-1](last_hidden_state).float(), torch.float32)
        w = torch.softmax(self.fusion_weights, dim=0)
        fused = None
        for i, (s, proj) in enumerate(zip(states, self.level_projs)):
            t = w[i] * proj(s).float()
            fused = t if fused is None else fused + t
        return self.norm(fused, torch.float32)
