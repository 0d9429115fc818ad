"""Reward model and verifiable rewards (reference: training/reward_model.py:21-135).

``RewardModel`` = Qwen3 backbone (no lm_head) + a scalar value head applied to
the last non-padding token; Bradley-Terry preference loss.  The backbone is
the same fused model; since the LM head is unused, only ``hidden`` runs.
``VerifiableReward`` scores math answers (\\boxed{}, '####' or last number)
and, for code, runs nothing: it checks that the reference answer appears in the
response, as the reference's placeholder does.
"""

from __future__ import annotations

import re
from typing import List, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..config import ModelConfig
from ..models.layers import Linear, fused_linear
from ..models.transformer import Qwen3Model


class RewardModel(nn.Module):
    def __init__(self, config: ModelConfig):
        super().__init__()
        self.backbone = Qwen3Model(config)
        self.value_head = Linear(config.hidden_size, 1, bias=False)
        nn.init.normal_(self.value_head.weight, std=config.initializer_range)

    def forward(self, input_ids: torch.Tensor, attention_mask: Optional[torch.Tensor] = None):
        x, _, _ = self.backbone.hidden(input_ids)
        B = x.shape[0]
        if attention_mask is not None:
            last = attention_mask.long().sum(-1) - 1
        else:
            last = torch.full((B,), x.shape[1] - 1, device=x.device, dtype=torch.long)
        pooled = x[torch.arange(B, device=x.device), last.clamp(min=0)]
        return fused_linear(pooled.float(), [self.value_head], torch.float32).squeeze(-1)

    def compute_preference_loss(self, chosen_ids, rejected_ids, chosen_mask=None, rejected_mask=None) -> dict:
        rc = self.forward(chosen_ids, chosen_mask)
        rr = self.forward(rejected_ids, rejected_mask)
        loss = -F.logsigmoid(rc - rr).mean()
        return {"loss": loss, "accuracy": (rc > rr).float().mean(), "chosen_reward": rc.mean(),
                "rejected_reward": rr.mean()}


class VerifiableReward:
    def __init__(self):
        self.reward_fns = {"math": self._math_reward, "code": self._code_reward}

    def compute(self, responses: List[str], ground_truths: List[str], task_type: str = "math") -> torch.Tensor:
        fn = self.reward_fns.get(task_type, self._default_reward)
        return torch.tensor([fn(r, g) for r, g in zip(responses, ground_truths)], dtype=torch.float32)

    @staticmethod
    def _extract(text: str) -> str:
        boxed = re.findall(r"\\boxed\{([^}]+)\}", text)
        if boxed:
            return boxed[-1].strip()
        nums = re.findall(r"-?\d+\.?\d*", text)
        return nums[-1] if nums else ""

    @classmethod
    def _math_reward(cls, response: str, ground_truth: str) -> float:
        p, g = cls._extract(response), cls._extract(ground_truth)
        try:
            return 1.0 if abs(float(p) - float(g)) < 1e-6 else 0.0
        except (ValueError, ZeroDivisionError):
            return 1.0 if p == g else 0.0

    @staticmethod
    def _code_reward(response: str, ground_truth: str) -> float:
        return 1.0 if ground_truth.strip() in response else 0.0

    @staticmethod
    def _default_reward(response: str, ground_truth: str) -> float:
        return 1.0 if ground_truth.strip() in response else 0.0
