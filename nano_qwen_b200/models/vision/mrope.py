"""Multimodal RoPE (temporal / height / width position components).

``MultimodalRoPE`` keeps the reference's API (three rotary tables of
head_dim/3 each, concatenated; reference: model/vision/mrope.py:18-65) and
``build_mrope_position_ids`` its semantics (text tokens keep their 1-D position
in all three components, image tokens get (t, h, w) grid coordinates;
reference: model/vision/mrope.py:68-120) without the per-token Python loops.

Unlike the reference (where MRoPE was never wired into attention),
``mrope_tables`` produces per-token cos/sin rows [B*S, D/2] that the fused
QK-norm/RoPE kernel consumes directly: the D/2 rotation frequencies are split
into sections (``mrope_section``; the head_dim/3 split of the reference by
default, or e.g. [16, 24, 24] for head_dim 128) and each section rotates by its
own position component.
"""

from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import torch
import torch.nn as nn

from ..rope import RotaryEmbedding, inv_freq_plain


class MultimodalRoPE(nn.Module):
    def __init__(self, head_dim: int, max_position_embeddings: int = 32768, base: float = 1e6):
        super().__init__()
        assert head_dim % 3 == 0, f"head_dim={head_dim} must be divisible by 3 for MRoPE"
        self.head_dim = head_dim
        self.section_dim = head_dim // 3
        self.rope_t = RotaryEmbedding(self.section_dim, max_position_embeddings, base)
        self.rope_h = RotaryEmbedding(self.section_dim, max_position_embeddings, base)
        self.rope_w = RotaryEmbedding(self.section_dim, max_position_embeddings, base)

    def forward(self, x, position_ids_t=None, position_ids_h=None, position_ids_w=None):
        ct, st = self.rope_t(x, position_ids_t)
        ch, sh = self.rope_h(x, position_ids_h)
        cw, sw = self.rope_w(x, position_ids_w)
        return torch.cat([ct, ch, cw], -1), torch.cat([st, sh, sw], -1)


def build_mrope_position_ids(text_positions: torch.Tensor, image_grid_thw: Optional[torch.Tensor] = None,
                             image_token_mask: Optional[torch.Tensor] = None):
    """(pos_t, pos_h, pos_w) each [B, S]; image tokens (in order, image after
    image) get their (t, h, w) grid coordinates."""
    pos_t = text_positions.clone()
    pos_h = text_positions.clone()
    pos_w = text_positions.clone()
    if image_grid_thw is None or image_token_mask is None:
        return pos_t, pos_h, pos_w
    coords = []
    for t, h, w in image_grid_thw.tolist():
        tt, hh, ww = torch.meshgrid(torch.arange(int(t)), torch.arange(int(h)), torch.arange(int(w)),
                                    indexing="ij")
        coords.append(torch.stack([tt.reshape(-1), hh.reshape(-1), ww.reshape(-1)], 1))
    grid = torch.cat(coords, 0).to(text_positions.device) if coords else None
    for b in range(text_positions.shape[0]):
        idx = image_token_mask[b].nonzero(as_tuple=True)[0]
        n = min(idx.numel(), grid.shape[0]) if grid is not None else 0
        if n == 0:
            continue
        pos_t[b, idx[:n]] = grid[:n, 0].to(pos_t.dtype)
        pos_h[b, idx[:n]] = grid[:n, 1].to(pos_h.dtype)
        pos_w[b, idx[:n]] = grid[:n, 2].to(pos_w.dtype)
    return pos_t, pos_h, pos_w


def mrope_tables(head_dim: int, base: float, pos_thw: Sequence[torch.Tensor],
                 sections: Optional[List[int]] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Per-token fp32 cos/sin rows [B*S, head_dim/2] for the fused RoPE kernel."""
    half = head_dim // 2
    if sections is None:
        sec = head_dim // 3
        sections = [sec // 2, sec // 2, half - 2 * (sec // 2)]
    assert sum(sections) == half, "mrope sections must sum to head_dim/2"
    pos_t, pos_h, pos_w = [p.reshape(-1).float() for p in pos_thw]
    inv = inv_freq_plain(head_dim, base).to(pos_t.device)
    which = torch.cat([torch.full((n,), i, dtype=torch.long) for i, n in enumerate(sections)]).to(pos_t.device)
    pos = torch.stack([pos_t, pos_h, pos_w], 1)[:, which]      # [T, half]
    ang = pos * inv[None, :]
    return ang.cos().contiguous(), ang.sin().contiguous()
