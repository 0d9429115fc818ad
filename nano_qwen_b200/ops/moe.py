"""Mixture-of-experts: router and the dropless / capacity expert FFN.

GPU design (no host synchronisation anywhere in the layer):

* ``router_fwd`` (one kernel): fp32 softmax over E, top-k, optional renorm,
  per-expert token counts and probability sums for the aux loss.
* ``moe_plan``: a stable counting sort of the N*k (token, slot) pairs by
  expert.  Each expert's rows start at a 128-row aligned offset of a buffer of
  static size N*k + E*128, so the grouped GEMMs need no host-side sizes and the
  weight-gradient GEMMs can run whole 128-row K blocks (padding rows are zero).
  Capacity mode drops the pairs whose rank inside their expert, in token order,
  is >= capacity (the reference's truncation order, model/moe.py:170-198).
* grouped tcgen05 GEMMs gate|up -> SwiGLU -> down over all experts in one
  launch each; the gather of token rows and the weighted top-k combine are
  separate bandwidth-bound kernels.

Replaces reference: model/moe.py:23-198 (a Python loop over experts with a
``nonzero`` host sync per expert) and kernels/moe_dispatch.py:22-64.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn.functional as F

from . import reference as ref
from ._ext import ext
from .linear import WeightRef

PAD = 128


# ----------------------------------------------------------------------------- router
class _RouterFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, top_k, norm_topk):
        E = ext()
        w, idx, counts, psum = E.router_fwd(logits, int(top_k), bool(norm_topk))
        ctx.save_for_backward(logits, w, idx, counts)
        ctx.norm = bool(norm_topk)
        ctx.mark_non_differentiable(idx, counts)
        return w, idx, counts, psum

    @staticmethod
    def backward(ctx, dw, didx, dcounts, dpsum):
        logits, w, idx, counts = ctx.saved_tensors
        if dw is None:
            dw = torch.zeros_like(w)
        if dpsum is None:
            dpsum = torch.zeros(counts.shape, dtype=torch.float32, device=logits.device)
        dlogits = ext().router_bwd(logits, w, idx, dw.contiguous(), dpsum.contiguous(), ctx.norm)
        return dlogits, None, None


def route(logits: torch.Tensor, top_k: int, norm_topk: bool):
    """Returns (weights fp32 [N,k], indices int32 [N,k], counts fp32 [E], prob_sum fp32 [E]).

    ``prob_sum`` is differentiable; aux = E * sum(counts/(N*k) * prob_sum/N).
    """
    if logits.is_cuda:
        return _RouterFn.apply(logits, top_k, norm_topk)
    w, idx, probs = ref.router(logits, top_k, norm_topk)
    E = logits.shape[-1]
    counts = torch.bincount(idx.reshape(-1), minlength=E).float()
    return w, idx.int(), counts, probs.sum(0)


def aux_loss_from_stats(counts: torch.Tensor, prob_sum: torch.Tensor, num_tokens: int,
                        top_k: int, num_experts: int,
                        global_counts: Optional[torch.Tensor] = None,
                        global_tokens: Optional[int] = None) -> torch.Tensor:
    """Switch-style aux loss E * sum_i f_i * p_i (reference: model/moe.py:63-89).

    With ``global_counts`` (summed over data-parallel ranks / micro-batches) the
    routing fractions f_i are global-batch statistics, which is the Qwen3
    global-batch balancing the reference describes (model/moe.py:201-249).
    """
    if global_counts is not None:
        f = global_counts / (global_tokens * top_k)
    else:
        f = counts / (num_tokens * top_k)
    p = prob_sum / num_tokens
    return num_experts * (f.detach() * p).sum()


# ------------------------------------------------------------------------ expert FFN
class _MoEFFNFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weights, idx, w_gu: WeightRef, w_d: WeightRef, num_experts, inter,
                capacity, *anchors):
        E = ext()
        N, H = x.shape
        k = idx.shape[1]
        # slot_of [N,k] int32: row of each (token, slot) pair in the expert-sorted
        # buffer, -1 when dropped; offsets [E+1] int32: aligned start row per expert.
        # src_of [N*k + E*PAD] int32: source token of each buffer row (-1 = zero row).
        slot_of, offsets, src_of = E.moe_plan(idx, num_experts, capacity, PAD)
        xp = E.moe_gather(x, src_of)
        Wgu = w_gu.compute.view(num_experts, 2 * inter, H)
        Wd = w_d.compute.view(num_experts, H, inter)
        gu = E.grouped_gemm_nt(xp, Wgu, offsets)
        h = E.swiglu_fwd(gu)
        y = E.grouped_gemm_nt(h, Wd, offsets)
        out = E.moe_combine(y, slot_of, weights)
        ctx.save_for_backward(x, weights, slot_of, offsets, xp, gu, h, y)
        ctx.w = (w_gu, w_d)
        ctx.meta = (num_experts, inter, len(w_gu.anchors))
        return out

    @staticmethod
    def backward(ctx, dout):
        x, weights, slot_of, offsets, xp, gu, h, y = ctx.saved_tensors
        w_gu, w_d = ctx.w
        num_experts, inter, n_gu = ctx.meta
        E = ext()
        N, H = x.shape
        dout = dout.contiguous()
        dy, dweights = E.moe_combine_bwd(dout, y, slot_of, weights)
        Wgu = w_gu.compute.view(num_experts, 2 * inter, H)
        Wd = w_d.compute.view(num_experts, H, inter)
        if w_d.requires_grad:
            E.grouped_gemm_tn_acc(dy, h, _grad_view(w_d, (num_experts, H, inter)), offsets)
        dh = E.grouped_gemm_nn(dy, Wd, offsets)
        dgu = E.swiglu_bwd(dh, gu)
        if w_gu.requires_grad:
            E.grouped_gemm_tn_acc(dgu, xp, _grad_view(w_gu, (num_experts, 2 * inter, H)), offsets)
        dxp = E.grouped_gemm_nn(dgu, Wgu, offsets)
        dx = E.moe_scatter_add(dxp, slot_of, N)
        return (dx, dweights, None, None, None, None, None, None) + \
            (None,) * (len(w_gu.anchors) + len(w_d.anchors))


def _grad_view(wref: WeightRef, shape):
    if wref.grad is None:
        raise RuntimeError("grouped expert weights must live in a FlatParamStore on GPU")
    return wref.grad.view(shape)


def moe_ffn(x: torch.Tensor, weights: torch.Tensor, idx: torch.Tensor, w_gu: WeightRef,
            w_d: WeightRef, num_experts: int, inter: int,
            capacity: Optional[int] = None) -> torch.Tensor:
    """x [N,H] routed to experts idx [N,k] with weights [N,k]; returns [N,H]."""
    if x.is_cuda:
        cap = -1 if capacity is None else int(capacity)
        return _MoEFFNFn.apply(x, weights, idx, w_gu, w_d, num_experts, inter, cap,
                               *w_gu.anchors, *w_d.anchors)
    return _moe_ffn_cpu(x, weights, idx, w_gu, w_d, num_experts, inter, capacity)


def _moe_ffn_cpu(x, weights, idx, w_gu, w_d, num_experts, inter, capacity):
    """Expert loop (the reference's algorithm) with weights routed through
    WeightRef so gradients land in the experts' gradient buffers."""
    from .linear import linear

    N, H = x.shape
    out = torch.zeros_like(x)
    idx = idx.long()
    gu_all = w_gu.compute.view(num_experts, 2 * inter, H)
    d_all = w_d.compute.view(num_experts, H, inter)
    for e in range(num_experts):
        mask = idx == e
        tok, slot = mask.nonzero(as_tuple=True)
        if tok.numel() == 0:
            continue
        if capacity is not None and tok.numel() > capacity:
            tok, slot = tok[:capacity], slot[:capacity]
        xe = x[tok]
        gu = linear(xe, _expert_ref(w_gu, gu_all, e))
        g, u = gu.chunk(2, dim=-1)
        he = F.silu(g) * u
        ye = linear(he, _expert_ref(w_d, d_all, e))
        out = out.index_add(0, tok, ye * weights[tok, slot].unsqueeze(-1).to(ye.dtype))
    return out


def _expert_ref(wref: WeightRef, stacked: torch.Tensor, e: int) -> WeightRef:
    """WeightRef of expert ``e``'s rows inside a stacked WeightRef."""
    n_rows = stacked.shape[1]
    per = len(wref.anchors) // stacked.shape[0]
    anchors = wref.anchors[e * per:(e + 1) * per]
    grad = None
    if wref.grad is not None:
        # sliced when the backward runs (the buffer may not be allocated yet)
        def grad():
            return wref.grad.view(stacked.shape)[e]
    return WeightRef(stacked[e], grad, anchors, parts=None if grad is not None else True)
