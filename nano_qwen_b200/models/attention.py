"""Grouped-query attention with QK-RMSNorm and RoPE (Qwen3).

Parameters and names follow the reference (q_proj/k_proj/v_proj/o_proj,
q_norm/k_norm; reference: model/attention.py:49-80).  Execution differs:

* training / full-sequence path: one GEMM over the contiguous q|k|v weight,
  then ``ops.attention_core`` (fused QK-norm + RoPE + flash attention), then
  o_proj;
* cached path (prefill and decode): positions continue from the cache length
  (the reference restarts RoPE at 0 on each decode step,
  reference: eval/generate.py:126-135 with model/rope.py:123-126) and
  prefill is causal (the reference runs cached prefill without a mask,
  model/attention.py:113).
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from .. import ops
from ..config import ModelConfig
from .kv_cache import KVCache
from .layers import Linear, RMSNorm, fused_linear
from .rope import RotaryEmbedding


class Attention(nn.Module):
    def __init__(self, config: ModelConfig, layer_idx: int = 0):
        super().__init__()
        self.config = config
        self.layer_idx = layer_idx
        self.hidden_size = config.hidden_size
        self.num_heads = config.num_attention_heads
        self.num_kv_heads = config.num_key_value_heads
        self.head_dim = config.head_dim
        self.num_kv_groups = config.num_kv_groups
        b = config.attention_bias
        self.q_proj = Linear(self.hidden_size, self.num_heads * self.head_dim, b)
        self.k_proj = Linear(self.hidden_size, self.num_kv_heads * self.head_dim, b)
        self.v_proj = Linear(self.hidden_size, self.num_kv_heads * self.head_dim, b)
        self.o_proj = Linear(self.num_heads * self.head_dim, self.hidden_size, b)
        self.qk_norm = config.qk_norm
        if self.qk_norm:
            self.q_norm = RMSNorm(self.head_dim, eps=config.rms_norm_eps)
            self.k_norm = RMSNorm(self.head_dim, eps=config.rms_norm_eps)
        self.rotary_emb = RotaryEmbedding(self.head_dim, config.max_position_embeddings,
                                          config.rope_theta, config.rope_scaling)
        # Tensor-parallel attention runs local heads only (set by parallel.tensor_parallel).
        self.tp_heads = None

    def fusion_groups(self):
        return [["q_proj.weight", "k_proj.weight", "v_proj.weight"]]

    def _heads(self):
        if self.tp_heads is not None:
            return self.tp_heads
        return self.num_heads, self.num_kv_heads

    def forward(self, hidden_states: torch.Tensor, position_ids: Optional[torch.Tensor] = None,
                attention_mask: Optional[torch.Tensor] = None,
                kv_cache: Optional[KVCache] = None, rope=None) -> torch.Tensor:
        """``rope`` = optional (cos, sin) per-token tables [B*S, D/2] (multimodal
        RoPE); they replace the 1-D position tables for this call."""
        B, S, _ = hidden_states.shape
        Hq, Hk = self._heads()
        D = self.head_dim
        dtype = hidden_states.dtype
        qkv = fused_linear(hidden_states, [self.q_proj, self.k_proj, self.v_proj], dtype)
        qw = self.q_norm.weight if self.qk_norm else None
        kw = self.k_norm.weight if self.qk_norm else None
        cos, sin = self.rotary_emb.cos_cached, self.rotary_emb.sin_cached
        if rope is not None:
            cos, sin = rope
            position_ids = torch.arange(B * S, device=qkv.device).view(B, S)
        eps = self.config.rms_norm_eps
        cp = getattr(self, "cp_group", None)
        if cp is not None and kv_cache is None:
            o = self._attend_cp(qkv, qw, kw, cos, sin, position_ids, B, S, Hq, Hk, D, eps, cp)
        elif kv_cache is None and (attention_mask is None or isinstance(attention_mask, ops.KeyRange)):
            # plain causal, or causal within per-token key ranges (packed
            # documents, padding) on the same kernels
            o = ops.attention_core(qkv, qw, kw, cos, sin, position_ids, Hq, Hk, D, eps,
                                   causal=True, key_range=attention_mask)
        else:
            o = self._attend_general(qkv, qw, kw, cos, sin, position_ids, attention_mask,
                                     kv_cache, B, S, Hq, Hk, D, eps)
        return fused_linear(o, [self.o_proj], dtype)

    def _attend_cp(self, qkv, qw, kw, cos, sin, position_ids, B, S, Hq, Hk, D, eps, group):
        """Context-parallel attention: local queries against the group's keys
        (``parallel.context_parallel.cp_attention``); positions are global."""
        from ..parallel.context_parallel import cp_attention, cp_attention_kernel, kernel_usable
        if getattr(self, "cp_mode", "allgather") == "ring":
            # k|v blocks passed around the ring: two blocks per rank in memory
            from ..parallel.ring_attention import ring_attention_qkv
            pos = position_ids.expand(B, S)
            return ring_attention_qkv(qkv, qw, kw, cos, sin, pos, group, Hq, Hk, D, eps)
        if qkv.is_cuda and kernel_usable(S):
            pos = position_ids.expand(B, S).to(torch.int64)
            return cp_attention_kernel(qkv, qw, kw, cos, sin, pos, group, Hq, Hk, D, eps,
                                       layer=self.layer_idx)
        q, k, v = qkv.split([Hq * D, Hk * D, Hk * D], dim=-1)
        q = q.reshape(B, S, Hq, D)
        k = k.reshape(B, S, Hk, D)
        v = v.reshape(B, S, Hk, D)
        pos = position_ids.expand(B, S)
        q, k = ops.reference.qk_norm_rope(q, k, qw, kw, cos[pos], sin[pos], eps)
        o = cp_attention(q, k, v, pos, group)
        return o.reshape(B, S, Hq * D)

    def _attend_general(self, qkv, qw, kw, cos, sin, position_ids, attention_mask, kv_cache,
                        B, S, Hq, Hk, D, eps):
        past = kv_cache.seq_len if kv_cache is not None else 0
        if position_ids is None:
            position_ids = (torch.arange(S, device=qkv.device) + past).unsqueeze(0).expand(B, S)
        q, k, v = ops.rope_qk(qkv, Hq, Hk, D, qw, kw, cos, sin, position_ids, eps)
        if kv_cache is not None:
            k_all, v_all = kv_cache.append(k, v)
        else:
            k_all, v_all = k, v
        if attention_mask is not None:
            o = _masked_attention(q, k_all, v_all, attention_mask, past)
        elif q.is_cuda and past == 0:
            # prefill into an empty cache: the flash-attention kernel on the prompt
            o = ops.attention_core(qkv, qw, kw, cos, sin, position_ids, Hq, Hk, D, eps,
                                   causal=True).view(B, S, Hq, D)
        elif q.is_cuda:
            kb, vb = (kv_cache.buffers() if kv_cache is not None else (k_all, v_all))
            # the decode kernel holds at most 32 (q-head, row) pairs per kv head
            rows = max(1, 32 // (Hq // Hk))
            outs = []
            for s0 in range(0, S, rows):
                s1 = min(S, s0 + rows)
                n = torch.full((B,), past + s1, dtype=torch.int32, device=q.device)
                start = torch.full((B,), past + s0, dtype=torch.int32, device=q.device)
                outs.append(ops.decode_attention(q[:, s0:s1].contiguous(), kb, vb, n, start))
            o = outs[0] if len(outs) == 1 else torch.cat(outs, 1)
        else:
            o = ops.reference.attention(q, k_all, v_all, causal=True, q_offset=past)
        return o.reshape(B, S, Hq * D)


def _masked_attention(q, k, v, attention_mask, past):
    """Causal attention plus a key-padding / additive mask (general path)."""
    import math
    B, Sq, Hq, D = q.shape
    Sk, Hk = k.shape[1], k.shape[2]
    g = Hq // Hk
    qf = q.float().reshape(B, Sq, Hk, g, D)
    s = torch.einsum("bqhgd,bkhd->bhgqk", qf, k.float()) / math.sqrt(D)
    causal = torch.arange(Sk, device=q.device)[None, :] > (torch.arange(Sq, device=q.device)[:, None] + past)
    s = s.masked_fill(causal, float("-inf"))
    m = attention_mask
    if isinstance(m, ops.KeyRange):  # key ranges of the new rows (positions past..past+Sq)
        early = torch.arange(Sk, device=q.device)[None, None, :] < m.kv_lo[:, :, None]
        s = s.masked_fill(early[:, None, None, :, :], float("-inf"))
    elif m.dtype == torch.bool or m.dtype in (torch.int32, torch.int64):
        if m.dim() == 2:  # [B, Sk] key padding, 1 = keep
            s = s.masked_fill(~m.bool()[:, None, None, None, :], float("-inf"))
        else:
            s = s.masked_fill(~m.bool().reshape(B, 1, 1, Sq, Sk), float("-inf"))
    else:
        s = s + m.float().reshape(B, 1, 1, Sq, Sk) if m.dim() == 4 else s + m.float()
    p = torch.softmax(s, dim=-1).nan_to_num(0.0)
    o = torch.einsum("bhgqk,bkhd->bqhgd", p, v.float())
    return o.reshape(B, Sq, Hq, D).to(q.dtype)
