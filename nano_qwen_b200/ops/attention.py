"""Attention core: QK-RMSNorm + RoPE + causal GQA flash attention.

One autograd node covers ``qkv -> o``:

* ``qknorm_rope_fwd`` reads the fused q|k|v GEMM output [T, (Hq+2Hk)*D],
  applies per-head RMSNorm to q and k and the NeoX rotation, and writes q|k
  [T, (Hq+Hk)*D]; v is read in place from the GEMM output.
* ``attn_fwd`` is the sm_100a flash-attention kernel (tcgen05 MMAs with TMEM
  accumulators, TMA-fed K/V ring): native GQA (no ``repeat_interleave``), causal
  mask, fp32 LSE output.  Inputs are token-major [T, heads*D] so no transposes
  are needed anywhere in the block.
* the backward writes dv straight into the v slot of d(qkv) and the
  QK-norm/RoPE backward writes the q and k slots, so d(qkv) feeds the fused QKV
  dgrad GEMM without a concatenation.

Replaces reference: model/attention.py:82-118 (view/transpose, two RMSNorm
composites, RoPE composite, repeat_interleave, SDPA) and the unused reference
kernels/flash_attn.py:28-88 and kernels/rope.py:20-56.
"""

from __future__ import annotations

import math
from typing import Optional

import torch

from . import reference as ref
from ._ext import ext
from .common import grad_buffer


def _rope_tables(cos: torch.Tensor, sin: torch.Tensor, position_ids: Optional[torch.Tensor],
                 B: int, S: int):
    """Gather [B or 1, S, D/2] fp32 cos/sin for the CPU path."""
    if position_ids is None:
        return cos[:S].unsqueeze(0), sin[:S].unsqueeze(0)
    return cos[position_ids], sin[position_ids]


class KeyRange:
    """Causal attention restricted to a key range per query: query i of a row
    sees keys [kv_lo[i], i], and key j is seen by queries [j, q_hi[j]).  This
    expresses packed documents (each token sees its own document only) and
    left or right padding, with ``kv_lo`` and ``q_hi`` non-decreasing along a
    row, so the attention kernels skip whole blocks outside the range.
    Tensors are int32 [B, S] on the device of the activations."""

    def __init__(self, kv_lo: torch.Tensor, q_hi: torch.Tensor):
        self.kv_lo = kv_lo.to(torch.int32).contiguous()
        self.q_hi = q_hi.to(torch.int32).contiguous()

    @classmethod
    def from_segments(cls, seg: torch.Tensor) -> "KeyRange":
        """``seg`` [B, S]: a segment (document) id per token, constant inside a
        segment, changing only at segment boundaries."""
        B, S = seg.shape
        idx = torch.arange(S, device=seg.device).expand(B, S)
        change = seg[:, 1:] != seg[:, :-1]
        first = torch.ones(B, S, dtype=torch.bool, device=seg.device)
        first[:, 1:] = change
        last = torch.ones(B, S, dtype=torch.bool, device=seg.device)
        last[:, :-1] = change
        kv_lo = torch.cummax(torch.where(first, idx, 0), dim=1).values
        ends = torch.where(last, idx + 1, S)
        q_hi = torch.flip(torch.cummin(torch.flip(ends, [1]), dim=1).values, [1])
        return cls(kv_lo, q_hi)

    @classmethod
    def from_padding_mask(cls, mask: torch.Tensor) -> Optional["KeyRange"]:
        """[B, S] key-padding mask (1 = real token) whose real tokens form one
        run per row (left or right padding): every token sees its own run.
        Returns None for other masks (reads the mask on the host once)."""
        m = mask.bool()
        run_starts = m.clone()
        run_starts[:, 1:] &= ~m[:, :-1]
        if int(run_starts.sum(1).max()) > 1:  # real tokens split into several runs
            return None
        return cls.from_segments(torch.cumsum(torch.cat([m[:, :1], m[:, 1:] != m[:, :-1]], 1).int(), 1))

    def numel(self) -> int:
        return self.kv_lo.numel()


class _AttnCoreFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, q_w, k_w, cos, sin, position_ids, Hq, Hk, D, eps, causal, scale, kv_lo, q_hi):
        B, S, W = qkv.shape
        qkv2 = qkv.reshape(B * S, W)
        E = ext()
        qk, rstd = E.qknorm_rope_fwd(qkv2, q_w, k_w, cos, sin, position_ids, B, S, Hq, Hk, D,
                                     float(eps))
        o, lse = E.attn_fwd(qk, qkv2, B, S, Hq, Hk, D, bool(causal), float(scale), kv_lo)
        ctx.save_for_backward(qkv2, qk, o, lse, rstd, q_w, k_w, cos, sin, position_ids, q_hi)
        ctx.meta = (B, S, Hq, Hk, D, float(eps), bool(causal), float(scale))
        return o.view(B, S, Hq * D)

    @staticmethod
    def backward(ctx, do):
        qkv2, qk, o, lse, rstd, q_w, k_w, cos, sin, position_ids, q_hi = ctx.saved_tensors
        B, S, Hq, Hk, D, eps, causal, scale = ctx.meta
        E = ext()
        do2 = do.reshape(B * S, Hq * D)
        if not do2.is_contiguous():
            do2 = do2.contiguous()
        dqkv = torch.empty_like(qkv2)
        dqk = E.attn_bwd(do2, qk, qkv2, o, lse, dqkv, B, S, Hq, Hk, D, causal, scale, q_hi)
        dqw = grad_buffer(q_w) if (q_w is not None and q_w.requires_grad) else None
        dkw = grad_buffer(k_w) if (k_w is not None and k_w.requires_grad) else None
        E.qknorm_rope_bwd(dqk, qkv2, q_w, k_w, rstd, cos, sin, position_ids, dqkv, dqw, dkw,
                          B, S, Hq, Hk, D)
        return (dqkv.view(B, S, -1),) + (None,) * 13


def attention_core(qkv: torch.Tensor, q_w: Optional[torch.Tensor], k_w: Optional[torch.Tensor],
                   cos: torch.Tensor, sin: torch.Tensor, position_ids: Optional[torch.Tensor],
                   num_heads: int, num_kv_heads: int, head_dim: int, eps: float,
                   causal: bool = True, scale: Optional[float] = None,
                   key_range: Optional[KeyRange] = None) -> torch.Tensor:
    """qkv [B, S, (Hq+2Hk)*D] -> attention output [B, S, Hq*D]; ``key_range``
    restricts each query's keys (document packing, padding)."""
    scale = scale if scale is not None else 1.0 / math.sqrt(head_dim)
    B, S, _ = qkv.shape
    Hq, Hk, D = num_heads, num_kv_heads, head_dim
    if qkv.is_cuda:
        lo = key_range.kv_lo.reshape(-1) if key_range is not None else None
        hi = key_range.q_hi.reshape(-1) if key_range is not None else None
        return _AttnCoreFn.apply(qkv, q_w, k_w, cos, sin, position_ids, Hq, Hk, D, eps, causal,
                                 scale, lo, hi)
    q, k, v = qkv.split([Hq * D, Hk * D, Hk * D], dim=-1)
    q = q.reshape(B, S, Hq, D)
    k = k.reshape(B, S, Hk, D)
    v = v.reshape(B, S, Hk, D)
    c, s = _rope_tables(cos, sin, position_ids, B, S)
    q, k = ref.qk_norm_rope(q, k, q_w, k_w, c, s, eps)
    o = ref.attention(q, k, v, causal=causal, scale=scale,
                      kv_lo=key_range.kv_lo if key_range is not None else None)
    return o.reshape(B, S, Hq * D)


def rope_qk(qkv: torch.Tensor, num_heads: int, num_kv_heads: int, head_dim: int, q_w, k_w,
            cos, sin, position_ids, eps):
    """QK-norm + RoPE at explicit positions for the cached path (no autograd).

    qkv [B, S, (Hq+2Hk)*D] -> q [B,S,Hq,D], k [B,S,Hk,D], v [B,S,Hk,D].
    """
    B, S, _ = qkv.shape
    Hq, Hk, D = num_heads, num_kv_heads, head_dim
    if qkv.is_cuda:
        qkv2 = qkv.reshape(B * S, -1).contiguous()
        qk, _ = ext().qknorm_rope_fwd(qkv2, q_w, k_w, cos, sin, position_ids, B, S, Hq, Hk, D,
                                      float(eps))
        q = qk[:, :Hq * D].reshape(B, S, Hq, D)
        k = qk[:, Hq * D:].reshape(B, S, Hk, D)
        v = qkv2[:, (Hq + Hk) * D:].reshape(B, S, Hk, D)
        return q, k, v
    q, k, v = qkv.split([Hq * D, Hk * D, Hk * D], dim=-1)
    q = q.reshape(B, S, Hq, D)
    k = k.reshape(B, S, Hk, D)
    v = v.reshape(B, S, Hk, D)
    c, s = _rope_tables(cos, sin, position_ids, B, S)
    q, k = ref.qk_norm_rope(q, k, q_w, k_w, c, s, eps)
    return q, k, v


def decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                     cache_len: torch.Tensor, q_start: torch.Tensor,
                     scale: Optional[float] = None) -> torch.Tensor:
    """Attention of new queries against a preallocated KV cache.

    q [B, Sq, Hq, D]; caches [B, Smax, Hk, D]; ``cache_len`` [B] int32 is the
    number of valid cache rows (including the new ones); ``q_start`` [B] int32
    is the absolute position of q row 0 (causal within the new rows).
    Reference being replaced: ``KVCache`` torch.cat growth + SDPA
    (reference: model/attention.py:24-46, :110-115).
    """
    D = q.shape[-1]
    scale = scale if scale is not None else 1.0 / math.sqrt(D)
    if q.is_cuda:
        return ext().decode_attn(q, k_cache, v_cache, cache_len, q_start, float(scale))
    B, Sq, Hq, _ = q.shape
    outs = []
    for b in range(B):
        n = int(cache_len[b])
        off = int(q_start[b])
        outs.append(ref.attention(q[b:b + 1], k_cache[b:b + 1, :n], v_cache[b:b + 1, :n],
                                  causal=True, scale=scale, q_offset=off))
    return torch.cat(outs, 0)


def full_attention(q, k, v, causal: bool = False, scale: Optional[float] = None):
    """Plain attention on [B, S, H, D] tensors (ViT; non-causal)."""
    D = q.shape[-1]
    scale = scale if scale is not None else 1.0 / math.sqrt(D)
    if q.is_cuda:
        return _FullAttnFn.apply(q, k, v, causal, scale)
    return ref.attention(q, k, v, causal=causal, scale=scale)


class _FullAttnFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, causal, scale):
        B, S, H, D = q.shape
        Hk = k.shape[2]
        q2 = q.reshape(B * S, H * D).contiguous()
        kv = torch.cat([k.reshape(B * S, Hk * D), v.reshape(B * S, Hk * D)], dim=1).contiguous()
        qk = torch.cat([q2, kv[:, :Hk * D]], dim=1).contiguous()
        qkv = torch.cat([qk, kv[:, Hk * D:]], dim=1).contiguous()
        o, lse = ext().attn_fwd(qk, qkv, B, S, H, Hk, D, bool(causal), float(scale))
        ctx.save_for_backward(qk, qkv, o, lse)
        ctx.meta = (B, S, H, Hk, D, bool(causal), float(scale))
        return o.view(B, S, H, D)

    @staticmethod
    def backward(ctx, do):
        qk, qkv, o, lse = ctx.saved_tensors
        B, S, H, Hk, D, causal, scale = ctx.meta
        do2 = do.reshape(B * S, H * D).contiguous()
        dqkv = torch.empty_like(qkv)
        dqk = ext().attn_bwd(do2, qk, qkv, o, lse, dqkv, B, S, H, Hk, D, causal, scale)
        dq = dqk[:, :H * D].to(q_dtype(do)).reshape(B, S, H, D)
        dk = dqk[:, H * D:].to(q_dtype(do)).reshape(B, S, Hk, D)
        dv = dqkv[:, (H + Hk) * D:].reshape(B, S, Hk, D)
        return dq, dk, dv, None, None


def q_dtype(t):
    return t.dtype
