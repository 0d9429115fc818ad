"""Token embedding gather / scatter-add.

The forward gathers rows into the fp32 residual stream (the reference's
``nn.Embedding`` output is fp32, reference: model/embedding.py:15).  When the
table lives in a flat parameter store the rows come from its bf16 compute
copy, the same copy the tied lm_head GEMM reads, which is complete on every
rank after a sharded optimizer step (the fp32 master is only up to date in the
rank's own shard).  The backward scatter-adds fp32 row gradients into the
table's gradient buffer with vectorised atomics.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from ._ext import ext
from .common import grad_buffer


def _table(weight: torch.Tensor) -> torch.Tensor:
    store = getattr(weight, "_nq_store", None)
    if store is not None and store.compute is not None:
        return store.compute_of(weight)
    return weight


class _EmbeddingFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, weight):
        ids_c = ids.reshape(-1).contiguous()
        out = ext().embedding_fwd(ids_c, _table(weight))
        ctx.save_for_backward(ids_c, weight)
        return out.view(*ids.shape, weight.shape[1])

    @staticmethod
    def backward(ctx, dout):
        ids_c, weight = ctx.saved_tensors
        if weight.requires_grad:
            d2 = dout.reshape(-1, dout.shape[-1])
            if d2.dtype != torch.float32 or not d2.is_contiguous():
                d2 = d2.float().contiguous()
            ext().embedding_bwd(ids_c, d2, grad_buffer(weight))
        return None, None


def embedding(ids: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    if ids.is_cuda:
        if torch.is_grad_enabled() and weight.requires_grad:
            return _EmbeddingFn.apply(ids, weight)
        return ext().embedding_fwd(ids.reshape(-1).contiguous(), _table(weight)).view(
            *ids.shape, weight.shape[1])
    return F.embedding(ids, weight)
