"""Preallocated KV caches for generation.

``KVCache`` keeps the reference's per-layer API (``update``, ``seq_len``,
``reset``; reference: model/attention.py:24-46) but stores K/V token-major
[B, S_max, Hk, D] in a buffer that grows geometrically instead of a
``torch.cat`` per decode step (O(T) copies per token in the reference).
``StaticKVCache`` is the fixed-capacity variant used by the decode engine
(CUDA-graph friendly: shapes never change, lengths live on the device).
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch


class KVCache:
    def __init__(self, capacity: int = 0):
        self._k: Optional[torch.Tensor] = None
        self._v: Optional[torch.Tensor] = None
        self._len = 0
        self._capacity = capacity

    def _ensure(self, B, need, Hk, D, dtype, device):
        if self._k is not None and self._k.shape[1] >= need:
            return
        cap = max(need, 2 * (self._k.shape[1] if self._k is not None else 0), self._capacity, 64)
        k = torch.empty(B, cap, Hk, D, dtype=dtype, device=device)
        v = torch.empty(B, cap, Hk, D, dtype=dtype, device=device)
        if self._k is not None and self._len:
            k[:, :self._len] = self._k[:, :self._len]
            v[:, :self._len] = self._v[:, :self._len]
        self._k, self._v = k, v

    def append(self, k: torch.Tensor, v: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """k, v [B, S_new, Hk, D]; returns views of all cached rows."""
        B, S, Hk, D = k.shape
        self._ensure(B, self._len + S, Hk, D, k.dtype, k.device)
        self._k[:, self._len:self._len + S] = k
        self._v[:, self._len:self._len + S] = v
        self._len += S
        return self._k[:, :self._len], self._v[:, :self._len]

    def update(self, key: torch.Tensor, value: torch.Tensor):
        """Reference API: key/value [B, Hk, S, D]; returns [B, Hk, S_total, D] views."""
        k, v = self.append(key.transpose(1, 2), value.transpose(1, 2))
        return k.transpose(1, 2), v.transpose(1, 2)

    @property
    def key(self):
        return None if self._k is None else self._k[:, :self._len].transpose(1, 2)

    @property
    def value(self):
        return None if self._v is None else self._v[:, :self._len].transpose(1, 2)

    @property
    def seq_len(self) -> int:
        return self._len

    def buffers(self):
        return self._k, self._v

    def reset(self) -> None:
        self._len = 0


class StaticKVCache:
    """Fixed [B, S_max, Hk, D] cache with a device-side length per sequence."""

    def __init__(self, batch: int, max_len: int, num_kv_heads: int, head_dim: int,
                 dtype: torch.dtype, device):
        self.k = torch.zeros(batch, max_len, num_kv_heads, head_dim, dtype=dtype, device=device)
        self.v = torch.zeros_like(self.k)
        self.lengths = torch.zeros(batch, dtype=torch.int32, device=device)
        self.max_len = max_len

    def reset(self) -> None:
        self.lengths.zero_()
