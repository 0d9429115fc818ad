"""Plain-PyTorch statements of every op's math.

These functions are the CPU execution path and the fp32 oracle the CUDA
kernel tests compare against.  They restate the reference's math:

* RMSNorm: fp32 normalise, cast back, then multiply by the weight
  (reference: model/norm.py:17-22).
* RoPE: NeoX half-split rotation (reference: model/rope.py:133-161).
* GQA attention without materialising repeated K/V
  (reference: model/attention.py:82-118).
* SwiGLU (reference: model/ffn.py:26).
* Router: fp32 softmax -> top-k -> optional renorm, Switch aux loss
  (reference: model/moe.py:36-89).
* Cross-entropy with ignore_index=-100, mean over valid targets.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn.functional as F


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return y.to(x.dtype) * weight.to(x.dtype)


def rotate_half_neox(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [..., S, H, D]; cos/sin broadcastable to [..., S, 1, D/2]."""
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)


def qk_norm_rope(q: torch.Tensor, k: torch.Tensor, q_w: Optional[torch.Tensor],
                 k_w: Optional[torch.Tensor], cos: torch.Tensor, sin: torch.Tensor,
                 eps: float) -> Tuple[torch.Tensor, torch.Tensor]:
    """q [B,S,Hq,D], k [B,S,Hk,D]; cos/sin [B or 1, S, D/2] (fp32)."""
    if q_w is not None:
        q = rms_norm(q, q_w, eps)
        k = rms_norm(k, k_w, eps)
    c = cos.unsqueeze(-2).to(q.dtype)
    s = sin.unsqueeze(-2).to(q.dtype)
    return rotate_half_neox(q, c, s), rotate_half_neox(k, c, s)


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = True,
              scale: Optional[float] = None, q_offset: int = 0,
              kv_len: Optional[torch.Tensor] = None,
              kv_lo: Optional[torch.Tensor] = None) -> torch.Tensor:
    """GQA attention.  q [B,Sq,Hq,D], k/v [B,Sk,Hk,D] -> [B,Sq,Hq,D].

    ``q_offset`` is the absolute position of q row 0 (decode / chunked prefill):
    query i may attend key j iff j <= i + q_offset.  ``kv_len`` [B] masks keys
    at positions >= kv_len[b] (padded caches).  ``kv_lo`` [B, Sq] masks keys
    before kv_lo[b, i] for query i (document packing, left padding).
    """
    B, Sq, Hq, D = q.shape
    Sk, Hk = k.shape[1], k.shape[2]
    g = Hq // Hk
    scale = scale if scale is not None else 1.0 / math.sqrt(D)
    qf = q.float().view(B, Sq, Hk, g, D)
    s = torch.einsum("bqhgd,bkhd->bhgqk", qf, k.float()) * scale
    mask = torch.zeros(Sq, Sk, dtype=torch.bool, device=q.device)
    if causal:
        qi = torch.arange(Sq, device=q.device)[:, None] + q_offset
        kj = torch.arange(Sk, device=q.device)[None, :]
        mask = kj > qi
    s = s.masked_fill(mask, float("-inf"))
    if kv_len is not None:
        kj = torch.arange(Sk, device=q.device)
        pad = kj[None, :] >= kv_len[:, None]  # [B, Sk]
        s = s.masked_fill(pad[:, None, None, None, :], float("-inf"))
    if kv_lo is not None:
        kj = torch.arange(Sk, device=q.device)
        early = kj[None, None, :] < kv_lo.to(q.device)[:, :, None]  # [B, Sq, Sk]
        s = s.masked_fill(early[:, None, None, :, :], float("-inf"))
    p = torch.softmax(s, dim=-1)
    o = torch.einsum("bhgqk,bkhd->bqhgd", p, v.float())
    return o.reshape(B, Sq, Hq, D).to(q.dtype)


def attention_lse(q, k, v, causal=True, scale=None):
    """Returns (out, lse [B,Hq,Sq]) in fp32 for kernel checks."""
    B, Sq, Hq, D = q.shape
    Sk, Hk = k.shape[1], k.shape[2]
    g = Hq // Hk
    scale = scale if scale is not None else 1.0 / math.sqrt(D)
    kr = k.float().repeat_interleave(g, dim=2)
    vr = v.float().repeat_interleave(g, dim=2)
    s = torch.einsum("bqhd,bkhd->bhqk", q.float(), kr) * scale
    if causal:
        m = torch.triu(torch.ones(Sq, Sk, dtype=torch.bool, device=q.device), diagonal=1 + Sk - Sq)
        s = s.masked_fill(m, float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    p = torch.exp(s - lse[..., None])
    o = torch.einsum("bhqk,bkhd->bqhd", p, vr)
    return o, lse


def swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    return F.silu(gate) * up


def router(logits: torch.Tensor, top_k: int, norm_topk: bool):
    """logits [N,E] -> (weights fp32 [N,k], indices [N,k], probs fp32 [N,E])."""
    probs = torch.softmax(logits.float(), dim=-1)
    w, idx = torch.topk(probs, top_k, dim=-1)
    if norm_topk:
        w = w / w.sum(-1, keepdim=True)
    return w, idx, probs


def switch_aux_loss(probs: torch.Tensor, idx: torch.Tensor, num_experts: int) -> torch.Tensor:
    """L = E * sum_i f_i * p_i  (reference: model/moe.py:63-89)."""
    n, k = idx.shape
    counts = torch.bincount(idx.reshape(-1), minlength=num_experts).float()
    f = counts / (n * k)
    p = probs.mean(0)
    return num_experts * (f * p).sum()


def cross_entropy(logits: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
    return F.cross_entropy(logits.float().view(-1, logits.shape[-1]), labels.view(-1),
                           ignore_index=-100)


def layer_norm(x, weight, bias, eps=1e-5):
    return F.layer_norm(x, (x.shape[-1],), weight, bias, eps)


def gelu(x):
    return F.gelu(x)
