"""Learning-rate schedules: linear warmup + cosine, and warmup-stable-decay.

Same formulas and ``build_scheduler`` signature as the reference
(training/scheduler.py:11-109).  The reference ignores the training YAML's
``optimizer.min_lr`` and hard-codes a 0.1 ratio; ``build_scheduler`` here
accepts ``min_lr`` and derives the ratio from it when given (otherwise 0.1).
"""

from __future__ import annotations

import math

import torch
from torch.optim.lr_scheduler import LRScheduler


class WarmupCosineScheduler(LRScheduler):
    def __init__(self, optimizer, warmup_steps: int = 2000, total_steps: int = 100000,
                 min_lr_ratio: float = 0.1, last_epoch: int = -1):
        self.warmup_steps = warmup_steps
        self.total_steps = total_steps
        self.min_lr_ratio = min_lr_ratio
        super().__init__(optimizer, last_epoch)

    def lr_at(self, step: int, base: float) -> float:
        floor = base * self.min_lr_ratio
        if step < self.warmup_steps:
            return base * step / max(1, self.warmup_steps)
        if step >= self.total_steps:
            return floor
        frac = (step - self.warmup_steps) / max(1, self.total_steps - self.warmup_steps)
        return floor + 0.5 * (base - floor) * (1.0 + math.cos(math.pi * frac))

    def get_lr(self):
        return [self.lr_at(self.last_epoch, b) for b in self.base_lrs]


class WSDScheduler(LRScheduler):
    def __init__(self, optimizer, warmup_steps: int = 2000, stable_steps: int = 80000,
                 decay_steps: int = 18000, min_lr_ratio: float = 0.1, last_epoch: int = -1):
        self.warmup_steps = warmup_steps
        self.stable_steps = stable_steps
        self.decay_steps = decay_steps
        self.min_lr_ratio = min_lr_ratio
        self.total_steps = warmup_steps + stable_steps + decay_steps
        super().__init__(optimizer, last_epoch)

    def lr_at(self, step: int, base: float) -> float:
        floor = base * self.min_lr_ratio
        if step < self.warmup_steps:
            return base * step / max(1, self.warmup_steps)
        if step < self.warmup_steps + self.stable_steps:
            return base
        frac = min((step - self.warmup_steps - self.stable_steps) / max(1, self.decay_steps), 1.0)
        return base - (base - floor) * frac

    def get_lr(self):
        return [self.lr_at(self.last_epoch, b) for b in self.base_lrs]


def build_scheduler(optimizer, scheduler_type: str = "cosine", warmup_steps: int = 2000,
                    total_steps: int = 100000, min_lr_ratio: float = 0.1, min_lr=None,
                    **kwargs):
    if min_lr is not None:
        base = optimizer.param_groups[0]["lr"]
        if base > 0:
            min_lr_ratio = float(min_lr) / base
    if scheduler_type == "cosine":
        return WarmupCosineScheduler(optimizer, warmup_steps, total_steps, min_lr_ratio)
    if scheduler_type == "wsd":
        stable = kwargs.get("stable_steps", int(total_steps * 0.8))
        decay = total_steps - warmup_steps - stable
        return WSDScheduler(optimizer, warmup_steps, stable, decay, min_lr_ratio)
    raise ValueError(f"Unknown scheduler type: {scheduler_type}")
