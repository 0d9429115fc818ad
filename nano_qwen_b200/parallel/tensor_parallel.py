"""Tensor parallelism with sequence parallelism (Megatron layout).

q/k/v and gate/up are column-parallel (each rank owns Hq/tp, Hk/tp heads and
I/tp FFN columns), o_proj and down_proj row-parallel.  With sequence
parallelism the residual stream, norms and loss run on a 1/tp slice of the
sequence: a column-parallel GEMM's input is all-gathered along the sequence and
a row-parallel GEMM's output is reduce-scattered back (their autograd duals
are the opposite collectives).  Attention runs on the full sequence for the
rank's local heads, which fixes the reference's TP, whose attention viewed the
local shard with the global head count and crashed (reference:
model/attention.py:91-93 with distributed/tensor_parallel.py:43-47).
Parameters that stay replicated (norms, embeddings, lm_head, routers) get their
gradients summed over the TP group by ``sync_replicated_grads``.

The collectives here are NCCL (Gloo on CPU, emulated where Gloo lacks the
primitive).
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist
import torch.nn as nn

from .comm import is_dist


# ------------------------------------------------------------ collectives
def _backend(group) -> str:
    return dist.get_backend(group) if is_dist() else "none"


def all_gather_dim(x: torch.Tensor, dim: int, group) -> torch.Tensor:
    ws = dist.get_world_size(group)
    if ws == 1:
        return x
    xc = x.movedim(dim, 0).contiguous()
    if _backend(group) == "nccl":
        out = torch.empty((ws * xc.shape[0],) + xc.shape[1:], dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(out, xc, group=group)
    else:
        parts = [torch.empty_like(xc) for _ in range(ws)]
        dist.all_gather(parts, xc, group=group)
        out = torch.cat(parts, 0)
    return out.movedim(0, dim)


def reduce_scatter_dim(x: torch.Tensor, dim: int, group) -> torch.Tensor:
    ws = dist.get_world_size(group)
    if ws == 1:
        return x
    xc = x.movedim(dim, 0).contiguous()
    n = xc.shape[0] // ws
    if _backend(group) == "nccl":
        out = torch.empty((n,) + xc.shape[1:], dtype=x.dtype, device=x.device)
        dist.reduce_scatter_tensor(out, xc, group=group)
    else:
        dist.all_reduce(xc, group=group)
        r = dist.get_rank(group)
        out = xc[r * n:(r + 1) * n].clone()
    return out.movedim(0, dim)


def split_dim(x: torch.Tensor, dim: int, group) -> torch.Tensor:
    ws = dist.get_world_size(group)
    if ws == 1:
        return x
    r = dist.get_rank(group)
    return x.chunk(ws, dim=dim)[r].contiguous()


class _GatherSeq(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return all_gather_dim(x, 1, group)

    @staticmethod
    def backward(ctx, g):
        return reduce_scatter_dim(g, 1, ctx.group), None


class _ScatterSeq(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return reduce_scatter_dim(x, 1, group)

    @staticmethod
    def backward(ctx, g):
        return all_gather_dim(g, 1, ctx.group), None


class _SplitSeq(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return split_dim(x, 1, group)

    @staticmethod
    def backward(ctx, g):
        return all_gather_dim(g, 1, ctx.group), None


class _AllReduce(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        x = x.clone()
        if dist.get_world_size(group) > 1:
            dist.all_reduce(x, group=group)
        return x

    @staticmethod
    def backward(ctx, g):
        return g, None


class _CopyToTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return x

    @staticmethod
    def backward(ctx, g):
        g = g.clone()
        if dist.get_world_size(ctx.group) > 1:
            dist.all_reduce(g, group=ctx.group)
        return g, None


class _ScaleGrad(torch.autograd.Function):
    """Identity forward; multiplies the gradient by ``s``."""

    @staticmethod
    def forward(ctx, x, s):
        ctx.s = s
        return x.view_as(x)

    @staticmethod
    def backward(ctx, g):
        return g * ctx.s, None


def scale_grad(x, s: float):
    return x if s == 1.0 else _ScaleGrad.apply(x, s)


def gather_seq(x, group):
    return _GatherSeq.apply(x, group)


def scatter_seq(x, group):
    return _ScatterSeq.apply(x, group)


def split_seq(x, group):
    return _SplitSeq.apply(x, group)


def tp_input(x: torch.Tensor, lin) -> torch.Tensor:
    """Input side of a column-parallel GEMM."""
    if getattr(lin, "tp_sp", False):
        return gather_seq(x, lin.tp_group)
    return _CopyToTP.apply(x, lin.tp_group)


def tp_output(y: torch.Tensor, lin) -> torch.Tensor:
    """Output side of a row-parallel GEMM."""
    if getattr(lin, "tp_sp", False):
        return scatter_seq(y, lin.tp_group)
    return _AllReduce.apply(y, lin.tp_group)


# ----------------------------------------------------------------- apply
def _shard_rows(lin, rank: int, ws: int, group, sp: bool):
    n = lin.weight.shape[0] // ws
    lin.weight = nn.Parameter(lin.weight.data[rank * n:(rank + 1) * n].clone())
    if lin.bias is not None:
        lin.bias = nn.Parameter(lin.bias.data[rank * n:(rank + 1) * n].clone())
        lin.bias._tp_sharded = True
    lin.weight._tp_sharded = True
    lin.tp_mode, lin.tp_group, lin.tp_sp = "col", group, sp


def _shard_cols(lin, rank: int, ws: int, group, sp: bool):
    n = lin.weight.shape[1] // ws
    lin.weight = nn.Parameter(lin.weight.data[:, rank * n:(rank + 1) * n].clone())
    lin.weight._tp_sharded = True
    lin.tp_mode, lin.tp_group, lin.tp_sp = "row", group, sp


def apply_tensor_parallel(model: nn.Module, tp_group, sequence_parallel: bool = True,
                          fused: Optional[bool] = None) -> nn.Module:
    """Shard every transformer block of a Qwen3Model (or the LM of a VL model).

    ``fused`` (default: when usable) runs dense models on CUDA through
    ``parallel.tp_fused``: the sequence-parallel all-gathers and
    reduce-scatters happen inside the norm and GEMM kernels over NVLink peer
    memory instead of as NCCL collectives."""
    if hasattr(tp_group, "get_group"):  # a DeviceMesh, as in the reference's API
        tp_group = tp_group.get_group()
    ws = dist.get_world_size(tp_group)
    r = dist.get_rank(tp_group)
    lm = getattr(model, "language_model", model)
    cfg = lm.config
    if cfg.num_attention_heads % ws or cfg.num_key_value_heads % ws:
        raise ValueError("attention heads must divide by tp_size")
    for blk in lm.layers:
        att = blk.attention
        # q, k, v are fused in one GEMM: all three must be column shards of the same rank
        for lin in (att.q_proj, att.k_proj, att.v_proj):
            _shard_rows(lin, r, ws, tp_group, sequence_parallel)
        _shard_cols(att.o_proj, r, ws, tp_group, sequence_parallel)
        att.tp_heads = (cfg.num_attention_heads // ws, cfg.num_key_value_heads // ws)
        ff = blk.feed_forward
        if hasattr(ff, "experts"):
            for ex in ff.experts:
                _shard_rows(ex.ffn.gate_proj, r, ws, tp_group, False)
                _shard_rows(ex.ffn.up_proj, r, ws, tp_group, False)
                _shard_cols(ex.ffn.down_proj, r, ws, tp_group, False)
            ff.inter = cfg.moe_intermediate_size // ws
            ff.tp_group, ff.tp_sp = tp_group, sequence_parallel
            ff.router.grad_scale = 1.0 / ws
        else:
            _shard_rows(ff.gate_proj, r, ws, tp_group, sequence_parallel)
            _shard_rows(ff.up_proj, r, ws, tp_group, sequence_parallel)
            _shard_cols(ff.down_proj, r, ws, tp_group, sequence_parallel)
    lm.tp_group = tp_group
    lm.sp_group = tp_group if sequence_parallel else None
    _mark_replicated(model, sequence_parallel)
    if fused is None:
        from .peer_dp import symmetric_available
        from .tp_fused import usable
        fused = sequence_parallel and usable(model) and symmetric_available(tp_group)
    lm.tp_fused = bool(fused) and sequence_parallel
    return model


def _mark_replicated(lm: nn.Module, sp: bool) -> None:
    """Tag every replicated parameter with how its gradient combines over TP.

    ``sum``: each rank holds a partial gradient -- q/k-norm weights (local
    heads only), routers (the combine weights see only the rank's partial
    expert outputs, and the aux loss, identical on every rank, is
    back-propagated at 1/tp by the MoE layer), and under sequence parallelism
    everything that runs on the rank's sequence slice (norms, lm_head, the
    embedding, which is looked up for the local slice only).  ``none``: the
    gradient is already identical on every rank (without sequence parallelism
    the norms, embedding and lm_head see the full, identical sequence).
    """
    for name, p in lm.named_parameters():
        if getattr(p, "_tp_sharded", False):
            continue
        partial = sp or "q_norm" in name or "k_norm" in name or "router" in name
        p._tp_reduce = "sum" if partial else "none"


@torch.no_grad()
def sync_replicated_grads(model: nn.Module, group) -> None:
    """Sum the partial gradients of replicated parameters over the TP group
    (the ``sum``-tagged ones, see ``_mark_replicated``)."""
    if group is None or dist.get_world_size(group) == 1:
        return
    grads = [p.grad for p in model.parameters()
             if p.grad is not None and getattr(p, "_tp_reduce", "none") == "sum"]
    if not grads:
        return
    flat = torch.cat([g.reshape(-1).float() for g in grads])
    dist.all_reduce(flat, group=group)
    o = 0
    for g in grads:
        n = g.numel()
        g.copy_(flat[o:o + n].view_as(g))
        o += n


# Reference-compatible standalone layers (reference: distributed/tensor_parallel.py:62-106)
class ColumnParallelLinear(nn.Module):
    def __init__(self, in_features, out_features, bias=False, process_group=None):
        super().__init__()
        from ..models.layers import Linear
        ws = dist.get_world_size(process_group) if process_group is not None else 1
        assert out_features % ws == 0
        self.linear = Linear(in_features, out_features // ws, bias)
        self.process_group = process_group

    def forward(self, x):
        if self.process_group is not None:
            x = _CopyToTP.apply(x, self.process_group)
        return self.linear(x)


class RowParallelLinear(nn.Module):
    def __init__(self, in_features, out_features, bias=False, process_group=None):
        super().__init__()
        from ..models.layers import Linear
        ws = dist.get_world_size(process_group) if process_group is not None else 1
        assert in_features % ws == 0
        self.linear = Linear(in_features // ws, out_features, bias)
        self.process_group = process_group

    def forward(self, x):
        y = self.linear(x)
        if self.process_group is not None:
            y = _AllReduce.apply(y, self.process_group)
        return y
