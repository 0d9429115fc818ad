"""Fused lm_head + vocab-chunked cross-entropy.

Never materialises the full [T, V] logits.  Rows are processed in chunks of
``chunk_rows``: a tcgen05 GEMM writes a bf16 logits chunk, one kernel turns it
in place into the loss contribution and d(logits) = (softmax - onehot) * g, and
two GEMMs consume it immediately (dX chunk, and dW accumulated in fp32).  With
``reduction="mean"`` the gradient is formed during the forward (the scale
1/n_valid is known on the device; no host sync) and the backward only rescales
by the incoming gradient.  With ``reduction="none"`` (per-token log-probs for
DPO/GRPO) the backward recomputes each chunk.

Replaces reference: model/transformer.py:138-145 (full fp32 logits +
``F.cross_entropy``) and kernels/cross_entropy.py:22-117 (whose backward
materialised softmax and one-hot [BT, V]).
"""

from __future__ import annotations


import torch
import torch.nn.functional as F

from ._ext import ext
from .common import rows
from .linear import WeightRef

DEFAULT_CHUNK_ROWS = 8192


def _chunks(T: int, n: int):
    for s in range(0, T, n):
        yield s, min(T, s + n)


class _LinearCEMeanFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, labels, wref: WeightRef, chunk_rows, *anchors):
        E = ext()
        h2 = rows(h)
        lab = labels.reshape(-1).contiguous()
        T = h2.shape[0]
        W = wref.compute
        V = W.shape[0]
        need_dx = h.requires_grad
        need_dw = wref.requires_grad
        n_valid = E.ce_count_valid(lab)  # fp32 scalar tensor, clamp(min=1)
        loss_sum = torch.zeros((), dtype=torch.float32, device=h.device)
        dh = torch.empty_like(h2) if need_dx else None
        dw = torch.zeros(W.shape, dtype=torch.float32, device=h.device) if need_dw else None
        buf = torch.empty((min(chunk_rows, T), V), dtype=h2.dtype, device=h.device)
        for s, e in _chunks(T, chunk_rows):
            logits = buf[: e - s]
            E.gemm_nt_out(h2[s:e], W, logits)
            E.ce_fused_chunk(logits, lab[s:e], n_valid, loss_sum, need_dx or need_dw)
            if need_dx:
                E.gemm_nn_out(logits, W, dh[s:e])
            if need_dw:
                E.gemm_tn_acc(logits, h2[s:e], dw)
        ctx.wref = wref
        ctx.save_for_backward(dh, dw)
        ctx.shape = h.shape
        return loss_sum / n_valid

    @staticmethod
    def backward(ctx, g):
        dh, dw = ctx.saved_tensors
        wref: WeightRef = ctx.wref
        E = ext()
        dx = None
        if dh is not None:
            E.scale_inplace(dh, g)
            dx = dh.view(ctx.shape)
        if dw is not None:
            if wref.grad is not None:
                E.axpy_(wref.grad, dw, g)
            else:
                wref.accumulate(dw * g)
        return (dx, None, None, None) + (None,) * len(wref.anchors)


class _LinearCENoneFn(torch.autograd.Function):
    """Per-row losses (-log p(label)); the backward recomputes logits."""

    @staticmethod
    def forward(ctx, h, labels, wref: WeightRef, chunk_rows, *anchors):
        E = ext()
        h2 = rows(h)
        lab = labels.reshape(-1).contiguous()
        T = h2.shape[0]
        W = wref.compute
        lse = torch.empty(T, dtype=torch.float32, device=h.device)
        tgt = torch.empty(T, dtype=torch.float32, device=h.device)
        buf = torch.empty((min(chunk_rows, T), W.shape[0]), dtype=h2.dtype, device=h.device)
        for s, e in _chunks(T, chunk_rows):
            logits = buf[: e - s]
            E.gemm_nt_out(h2[s:e], W, logits)
            E.ce_lse_chunk(logits, lab[s:e], lse[s:e], tgt[s:e])
        ctx.wref = wref
        ctx.chunk_rows = chunk_rows
        ctx.save_for_backward(h2, lab, lse)
        ctx.shape = h.shape
        loss = lse - tgt
        loss = torch.where(lab == -100, torch.zeros_like(loss), loss)
        return loss.view(labels.shape)

    @staticmethod
    def backward(ctx, g):
        h2, lab, lse = ctx.saved_tensors
        wref: WeightRef = ctx.wref
        E = ext()
        W = wref.compute
        T = h2.shape[0]
        g = g.reshape(-1).float().contiguous()
        need_dx = ctx.needs_input_grad[0]
        dh = torch.empty_like(h2) if need_dx else None
        dw = None
        if wref.requires_grad:
            dw = wref.grad if wref.grad is not None else torch.zeros(W.shape, dtype=torch.float32,
                                                                     device=h2.device)
        buf = torch.empty((min(ctx.chunk_rows, T), W.shape[0]), dtype=h2.dtype, device=h2.device)
        for s, e in _chunks(T, ctx.chunk_rows):
            logits = buf[: e - s]
            E.gemm_nt_out(h2[s:e], W, logits)
            E.ce_grad_chunk(logits, lab[s:e], lse[s:e], g[s:e])
            if need_dx:
                E.gemm_nn_out(logits, W, dh[s:e])
            if dw is not None:
                E.gemm_tn_acc(logits, h2[s:e], dw)
        if dw is not None and wref.grad is None:
            wref.accumulate(dw)
        dx = dh.view(ctx.shape) if need_dx else None
        return (dx, None, None, None) + (None,) * len(wref.anchors)


def linear_cross_entropy(h: torch.Tensor, wref: WeightRef, labels: torch.Tensor,
                         reduction: str = "mean",
                         chunk_rows: int = DEFAULT_CHUNK_ROWS) -> torch.Tensor:
    """CE(h @ W^T, labels) with ignore_index=-100.

    ``labels`` are the targets of each row (already shifted by the caller).
    """
    if h.is_cuda:
        fn = _LinearCEMeanFn if reduction == "mean" else _LinearCENoneFn
        return fn.apply(h, labels, wref, chunk_rows, *wref.anchors)
    h2 = h.reshape(-1, h.shape[-1])
    if torch.is_grad_enabled() and wref.requires_grad:
        logits = _CPULinearFn.apply(h2, wref, *wref.anchors)
    else:
        logits = h2 @ wref.compute.t().to(h.dtype)
    loss = F.cross_entropy(logits.float(), labels.reshape(-1), ignore_index=-100,
                           reduction=reduction)
    return loss.view(labels.shape) if reduction == "none" else loss


class _CPULinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h2, wref, *anchors):
        ctx.save_for_backward(h2)
        ctx.wref = wref
        return h2 @ wref.compute.t().to(h2.dtype)

    @staticmethod
    def backward(ctx, dlogits):
        (h2,) = ctx.saved_tensors
        wref = ctx.wref
        w = wref.compute.to(dlogits.dtype)
        dx = dlogits @ w if ctx.needs_input_grad[0] else None
        if wref.requires_grad:
            wref.accumulate(dlogits.t().float() @ h2.float())
        return (dx, None) + (None,) * len(wref.anchors)


def token_logprobs(h: torch.Tensor, wref: WeightRef, targets: torch.Tensor,
                   temperature: float = 1.0) -> torch.Tensor:
    """log p(target | row) for every row, without materialising [T, V] on GPU."""
    if temperature != 1.0:
        h = h / temperature
    return -linear_cross_entropy(h, wref, targets, reduction="none")
