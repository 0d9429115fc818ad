"""The reference's standalone kernel entry points, on this framework's ops.

The reference ships six op modules (reference: kernels/cross_entropy.py,
kernels/flash_attn.py, kernels/moe_dispatch.py, kernels/rmsnorm.py,
kernels/rope.py, kernels/swiglu.py) whose public functions pick a Triton
kernel or a PyTorch fallback with ``use_triton``.  The same names and
signatures are kept here for callers of that API; ``use_triton`` is accepted
and has no effect.  On CUDA tensors the sm_100a kernels run where this
framework has one for the op (cross-entropy, flash attention, RMSNorm,
SwiGLU); RoPE and the top-k scatter / gather are written as PyTorch tensor
operations (the model itself runs them fused into the QK-norm kernel and the
MoE plan / grouped GEMMs).  CPU tensors run the PyTorch statement of each op.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops

__all__ = ["fused_cross_entropy", "flash_attention", "scatter_tokens", "gather_tokens",
           "rmsnorm", "FusedRMSNorm", "apply_rope", "fused_swiglu"]


# ----------------------------------------------------------- cross-entropy
class _CrossEntropyFn(torch.autograd.Function):
    """Mean cross-entropy of bf16 logits on the fused kernel: one pass per
    row gives the loss and, in place of a copy of the logits, the gradient
    (softmax - onehot) / n_valid."""

    @staticmethod
    def forward(ctx, logits, labels):
        E = ops.ext()
        V = logits.shape[-1]
        buf = logits.reshape(-1, V).to(torch.bfloat16, copy=True).contiguous()
        lab = labels.reshape(-1).contiguous()
        n_valid = E.ce_count_valid(lab)
        loss_sum = torch.zeros((), dtype=torch.float32, device=logits.device)
        E.ce_fused_chunk(buf, lab, n_valid, loss_sum, logits.requires_grad)
        ctx.save_for_backward(buf)
        ctx.shape, ctx.dtype = logits.shape, logits.dtype
        return loss_sum / n_valid

    @staticmethod
    def backward(ctx, g):
        (buf,) = ctx.saved_tensors
        return (buf.float() * g).to(ctx.dtype).view(ctx.shape), None


def fused_cross_entropy(logits: torch.Tensor, labels: torch.Tensor, ignore_index: int = -100,
                        use_triton: bool = True) -> torch.Tensor:
    """Mean cross-entropy over the rows whose label is not ``ignore_index``
    (``F.cross_entropy`` semantics); logits [N, V], labels [N]."""
    if logits.is_cuda and logits.shape[-1] % 8 == 0:
        if ignore_index != -100:
            labels = torch.where(labels == ignore_index, torch.full_like(labels, -100), labels)
        return _CrossEntropyFn.apply(logits, labels)
    return F.cross_entropy(logits.float(), labels, ignore_index=ignore_index)


# --------------------------------------------------------- flash attention
def flash_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = True,
                    sm_scale: Optional[float] = None, use_triton: bool = True) -> torch.Tensor:
    """q [B, H, S, D], k/v [B, Hk, S, D] (Hk dividing H: grouped-query heads)
    -> [B, H, S, D]; ``sm_scale`` defaults to 1/sqrt(D).  CUDA: the tcgen05
    flash-attention kernels (bf16, D of 64 or 128, forward and backward)."""
    D = q.shape[-1]
    scale = sm_scale if sm_scale is not None else D ** -0.5
    if q.is_cuda and D in (64, 128):
        dt = q.dtype
        o = ops.full_attention(q.transpose(1, 2).to(torch.bfloat16), k.transpose(1, 2).to(torch.bfloat16),
                               v.transpose(1, 2).to(torch.bfloat16), causal=causal, scale=scale)
        return o.transpose(1, 2).to(dt)
    g = q.shape[1] // k.shape[1]
    if g > 1:
        k = k.repeat_interleave(g, dim=1)
        v = v.repeat_interleave(g, dim=1)
    return F.scaled_dot_product_attention(q, k, v, is_causal=causal, scale=scale)


# -------------------------------------------------------------- MoE routing
def scatter_tokens(x: torch.Tensor, flat_indices: torch.Tensor, weights: torch.Tensor,
                   num_slots: int, use_triton: bool = True) -> torch.Tensor:
    """out[flat_indices[n, k]] += x[n] * weights[n, k]; x [N, D] -> [num_slots, D]."""
    N, D = x.shape
    out = torch.zeros(num_slots, D, dtype=x.dtype, device=x.device)
    for j in range(flat_indices.shape[1]):
        out = out.index_add(0, flat_indices[:, j].long(), x * weights[:, j:j + 1].to(x.dtype))
    return out


def gather_tokens(expert_out: torch.Tensor, flat_indices: torch.Tensor, weights: torch.Tensor,
                  num_tokens: int, D: int, use_triton: bool = True) -> torch.Tensor:
    """out[n] = sum_k expert_out[flat_indices[n, k]] * weights[n, k] -> [num_tokens, D]."""
    out = torch.zeros(num_tokens, D, dtype=expert_out.dtype, device=expert_out.device)
    for j in range(flat_indices.shape[1]):
        out = out + expert_out[flat_indices[:, j].long()] * weights[:, j:j + 1].to(expert_out.dtype)
    return out


# ------------------------------------------------------------------ RMSNorm
def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """RMSNorm over the last dimension (differentiable); CUDA: the fused
    kernel."""
    return ops.rms_norm(x, weight, eps)


class FusedRMSNorm(nn.Module):
    """RMSNorm module with the reference's constructor."""

    def __init__(self, hidden_size: int, eps: float = 1e-6, use_triton: bool = True):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden_size))
        self.eps = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return rmsnorm(x, self.weight, self.eps)


# --------------------------------------------------------------------- RoPE
def apply_rope(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
               use_triton: bool = True) -> Tuple[torch.Tensor, torch.Tensor]:
    """NeoX-style rotation of q/k [B, H, S, D] by cos/sin [S, D/2] or
    [B, S, D/2]."""
    if cos.dim() == 2:
        c, s = cos[None, None], sin[None, None]
    else:
        c, s = cos[:, None], sin[:, None]
    c, s = c.to(q.dtype), s.to(q.dtype)
    return (ops.reference.rotate_half_neox(q, c, s), ops.reference.rotate_half_neox(k, c, s))


# ------------------------------------------------------------------- SwiGLU
def fused_swiglu(gate: torch.Tensor, up: torch.Tensor, use_triton: bool = True) -> torch.Tensor:
    """silu(gate) * up; CUDA: the SwiGLU kernel (bf16) on [gate | up]."""
    if gate.is_cuda and gate.shape[-1] % 8 == 0:
        dt = gate.dtype
        gu = torch.cat([gate, up], dim=-1).to(torch.bfloat16)
        return ops.swiglu_packed(gu).to(dt)
    return F.silu(gate) * up
