"""Deterministic distributed sampler with resume offset.

Same behaviour and API as the reference (seeded permutation per epoch, pad to
a multiple of the world size, stride-shard by rank, ``start_index`` resume,
``state_dict``; reference: data/sampler.py:13-84).  The trainers save its
state in checkpoints (the reference never did).
"""

from __future__ import annotations

import math
from typing import Iterator

import numpy as np
from torch.utils.data import Sampler


class DistributedSampler(Sampler):
    def __init__(self, dataset, num_replicas: int = 1, rank: int = 0, shuffle: bool = True,
                 seed: int = 42, drop_last: bool = False, start_index: int = 0):
        self.dataset = dataset
        self.num_replicas = num_replicas
        self.rank = rank
        self.shuffle = shuffle
        self.seed = seed
        self.drop_last = drop_last
        self.start_index = start_index
        self.epoch = 0
        n = len(dataset)
        self.num_samples = n // num_replicas if drop_last else math.ceil(n / num_replicas)
        self.total_size = self.num_samples * num_replicas

    def __iter__(self) -> Iterator[int]:
        n = len(self.dataset)
        if self.shuffle:
            idx = np.random.RandomState(self.seed + self.epoch).permutation(n).tolist()
        else:
            idx = list(range(n))
        if len(idx) < self.total_size:
            idx += idx[: self.total_size - len(idx)]
        else:
            idx = idx[: self.total_size]
        idx = idx[self.rank::self.num_replicas]
        return iter(idx[self.start_index:])

    def __len__(self) -> int:
        return max(0, self.num_samples - self.start_index)

    def set_epoch(self, epoch: int) -> None:
        self.epoch = epoch

    def set_start_index(self, start_index: int) -> None:
        self.start_index = start_index

    def state_dict(self) -> dict:
        return {"epoch": self.epoch, "start_index": self.start_index}

    def load_state_dict(self, state: dict) -> None:
        self.epoch = state.get("epoch", 0)
        self.start_index = state.get("start_index", 0)
