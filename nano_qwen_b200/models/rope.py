"""Rotary position tables: plain RoPE with an adjustable base (ABF) and YARN.

The tables are fp32 [max_positions, head_dim/2] cos/sin buffers consumed by the
fused QK-norm/RoPE kernel.  YARN follows the reference's blend of interpolated
and extrapolated inverse frequencies with a linear ramp between the correction
dims for beta_fast=32 / beta_slow=1 (reference: model/rope.py:31-75).  As an
option (``rope_scaling["mscale"]=True``) the attention-temperature factor
0.1*ln(factor)+1 of the YARN paper is folded into the tables; the reference
omits it, so it is off by default.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn as nn


def inv_freq_plain(dim: int, base: float) -> torch.Tensor:
    return 1.0 / (base ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim))


def _correction_dim(rotations: float, dim: int, base: float, max_pos: int) -> float:
    return (dim * math.log(max_pos / (rotations * 2 * math.pi))) / (2 * math.log(base))


def yarn_inv_freq(dim: int, base: float, factor: float, original_max: int,
                  beta_fast: float = 32.0, beta_slow: float = 1.0) -> torch.Tensor:
    extrap = inv_freq_plain(dim, base)
    interp = extrap / factor
    lo = max(math.floor(_correction_dim(beta_fast, dim, base, original_max)), 0)
    hi = min(math.ceil(_correction_dim(beta_slow, dim, base, original_max)), dim - 1)
    if lo == hi:
        hi = hi + 0.001
    ramp = ((torch.arange(dim // 2, dtype=torch.float32) - lo) / (hi - lo)).clamp(0, 1)
    keep_extrap = 1.0 - ramp
    return interp * (1 - keep_extrap) + extrap * keep_extrap


def rope_tables(dim: int, max_positions: int, base: float,
                rope_scaling: Optional[dict] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    scale = 1.0
    if rope_scaling is not None and rope_scaling.get("type") == "yarn":
        factor = float(rope_scaling.get("factor", 4.0))
        orig = int(rope_scaling.get("original_max_position_embeddings", 32768))
        inv = yarn_inv_freq(dim, base, factor, orig,
                            float(rope_scaling.get("beta_fast", 32.0)),
                            float(rope_scaling.get("beta_slow", 1.0)))
        if rope_scaling.get("mscale", False) and factor > 1:
            scale = 0.1 * math.log(factor) + 1.0
    else:
        inv = inv_freq_plain(dim, base)
    t = torch.arange(max_positions, dtype=torch.float32)
    freqs = torch.outer(t, inv)
    return freqs.cos() * scale, freqs.sin() * scale


class RotaryEmbedding(nn.Module):
    """Holds the cos/sin tables (non-persistent buffers, as in the reference)."""

    def __init__(self, dim: int, max_position_embeddings: int = 32768, base: float = 1e6,
                 rope_scaling: Optional[dict] = None):
        super().__init__()
        self.dim = dim
        self.max_position_embeddings = max_position_embeddings
        self.base = base
        self.rope_scaling = rope_scaling
        cos, sin = rope_tables(dim, max_position_embeddings, base, rope_scaling)
        self.register_buffer("cos_cached", cos, persistent=False)
        self.register_buffer("sin_cached", sin, persistent=False)

    def forward(self, x: torch.Tensor, position_ids: Optional[torch.Tensor] = None):
        """(cos, sin) gathered for ``position_ids`` (reference API, model/rope.py:109-130)."""
        if position_ids is None:
            S = x.shape[-2]
            return self.cos_cached[:S].to(x.dtype), self.sin_cached[:S].to(x.dtype)
        return self.cos_cached[position_ids].to(x.dtype), self.sin_cached[position_ids].to(x.dtype)


def apply_rotary_pos_emb(q, k, cos, sin):
    """Reference-compatible helper on [B, H, S, D] tensors (model/rope.py:133-161)."""
    def rot(x, c, s):
        if c.dim() == 2:
            c, s = c[None, None], s[None, None]
        elif c.dim() == 3:
            c, s = c[:, None], s[:, None]
        h = x.shape[-1] // 2
        x1, x2 = x[..., :h], x[..., h:]
        return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)
    return rot(q, cos, sin), rot(k, cos, sin)
