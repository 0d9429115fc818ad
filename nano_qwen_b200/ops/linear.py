"""Linear layers whose weight gradient is accumulated straight into the
parameter's fp32 gradient buffer.

Design (B200): parameters live in one flat fp32 master buffer with a bf16
compute copy that the fused AdamW kernel refreshes after each update
(``runtime.flat_params``).  A layer that spans several parameters (q|k|v,
gate|up, all experts of an MoE layer) uses one contiguous view of both buffers,
so the forward is a single tcgen05 GEMM and the weight-gradient GEMM writes into
the gradient buffer with beta=1: no per-step casts, no ``torch.cat`` and no
AccumulateGrad traffic.  Reference behaviour being replaced: ``nn.Linear`` under
bf16 autocast (reference: model/attention.py:63-66, model/ffn.py:21-23,
training/pretrain.py:172).
"""

from __future__ import annotations

from typing import Optional, Sequence

import torch

from ._ext import ext


class WeightRef:
    """A (possibly fused) weight [N, K] as seen by one GEMM.

    ``compute``: tensor used in the forward GEMM (bf16 on CUDA).
    ``grad``: fp32 [N, K] buffer the weight-gradient GEMM accumulates into, or
    None when the rows belong to separate gradient tensors (``parts``).  It
    may be given as a zero-argument callable that returns the buffer, so a
    slice of a gradient buffer that only exists during the backward (fully
    sharded parameters) is taken when the backward needs it.
    ``anchors``: the leaf Parameters, passed through autograd so that outputs
    require grad; their autograd gradient is always None.
    """

    __slots__ = ("compute", "_grad", "anchors", "parts")

    def __init__(self, compute, grad, anchors, parts=None):
        self.compute = compute
        self._grad = grad
        self.anchors = tuple(anchors)
        self.parts = parts

    @property
    def grad(self):
        g = self._grad
        return g() if callable(g) else g

    @property
    def requires_grad(self) -> bool:
        return any(a.requires_grad for a in self.anchors)

    def accumulate(self, dw: torch.Tensor) -> None:
        """Add a full [N, K] gradient (used by the CPU path and the fallback
        for non-contiguous parts)."""
        if self.grad is not None:
            self.grad.add_(dw.to(self.grad.dtype))
            return
        row = 0
        for p in self.anchors:
            n = p.shape[0]
            if p.requires_grad:
                piece = dw[row:row + n].reshape(p.shape).to(p.dtype)
                if p.grad is None:
                    p.grad = piece.clone()
                else:
                    p.grad.add_(piece)
            row += n


def _store_of(p: torch.Tensor):
    return getattr(p, "_nq_store", None)


def weight_ref(params: Sequence[torch.Tensor], compute_dtype: torch.dtype) -> WeightRef:
    """Build the WeightRef for rows ``cat(params, 0)``.

    If every parameter lives contiguously in one ``FlatParamStore`` the views
    are zero-copy; otherwise the compute weight is concatenated on the fly.
    """
    params = list(params)
    store = _store_of(params[0])
    if store is not None and all(_store_of(p) is store for p in params):
        view = store.fused_view(params, compute_dtype)
        if view is not None:
            compute, grad = view
            return WeightRef(compute, grad, params)
    ws = [p if p.dim() == 2 else p.reshape(p.shape[0], -1) for p in params]
    compute = ws[0] if len(ws) == 1 else torch.cat(ws, 0)
    compute = compute.detach().to(compute_dtype)
    if len(params) == 1 and params[0].requires_grad and params[0].grad is not None \
            and params[0].grad.dtype == torch.float32 and params[0].dim() == 2:
        return WeightRef(compute, params[0].grad, params)
    return WeightRef(compute, None, params, parts=True)


class _LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, wref: WeightRef, *anchors):
        w = wref.compute
        x2 = x.reshape(-1, x.shape[-1])
        if x.is_cuda:
            y = ext().gemm_nt(x2, w)
        else:
            y = x2 @ w.t()
        ctx.wref = wref
        ctx.save_for_backward(x2)
        ctx.in_shape = x.shape
        return y.view(*x.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):
        (x2,) = ctx.saved_tensors
        dx = linear_backward(dy.reshape(-1, dy.shape[-1]), x2, ctx.wref, ctx.needs_input_grad[0], ctx.in_shape)
        return (dx, None) + (None,) * len(ctx.wref.anchors)


def linear_backward(dy2: torch.Tensor, x2: torch.Tensor, wref: WeightRef, need_dx: bool, in_shape):
    """dx = dy W (if ``need_dx``) and W.grad += dy^T x for y = x W^T."""
    w = wref.compute
    if not dy2.is_contiguous():
        dy2 = dy2.contiguous()
    dx = None
    if dy2.is_cuda:
        E = ext()
        if need_dx:
            dx = E.gemm_nn(dy2, w).view(in_shape)
        if wref.requires_grad:
            if wref.grad is not None:
                E.gemm_tn_acc(dy2, x2, wref.grad)
            else:
                dw = torch.zeros(w.shape, dtype=torch.float32, device=w.device)
                E.gemm_tn_acc(dy2, x2, dw)
                wref.accumulate(dw)
    else:
        if need_dx:
            dx = (dy2 @ w).view(in_shape)
        if wref.requires_grad:
            wref.accumulate(dy2.t().to(torch.float32) @ x2.to(torch.float32))
    return dx


class _DenseFn(torch.autograd.Function):
    """y = x W^T with both inputs ordinary autograd tensors (the weight gradient
    is returned, not accumulated in place); for weights derived by other ops."""

    @staticmethod
    def forward(ctx, x, w):
        x2 = x.reshape(-1, x.shape[-1]).contiguous()
        ctx.save_for_backward(x2, w)
        ctx.in_shape = x.shape
        y = ext().gemm_nt(x2, w.contiguous())
        return y.view(*x.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2, w = ctx.saved_tensors
        dy2 = dy.reshape(-1, dy.shape[-1]).contiguous()
        E = ext()
        dx = E.gemm_nn(dy2, w.contiguous()).view(ctx.in_shape) if ctx.needs_input_grad[0] else None
        dw = None
        if ctx.needs_input_grad[1]:
            dw = torch.zeros(w.shape, dtype=torch.float32, device=w.device)
            E.gemm_tn_acc(dy2, x2, dw)
            dw = dw.to(w.dtype)
        return dx, dw


def dense(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """x @ w^T through the tcgen05 GEMM with standard autograd semantics."""
    if x.is_cuda:
        return _DenseFn.apply(x, w)
    return x @ w.t()


def linear(x: torch.Tensor, wref: WeightRef, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    if torch.is_grad_enabled() and (x.requires_grad or wref.requires_grad):
        y = _LinearFn.apply(x, wref, *wref.anchors)
    else:
        w = wref.compute
        x2 = x.reshape(-1, x.shape[-1])
        y = ext().gemm_nt(x2, w) if x.is_cuda else x2 @ w.t()
        y = y.view(*x.shape[:-1], w.shape[0])
    if bias is not None:
        y = y + bias.to(y.dtype)
    return y
