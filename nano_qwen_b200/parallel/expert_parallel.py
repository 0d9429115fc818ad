"""Expert parallelism: each EP rank owns E/ep experts; tokens travel to the
rank that owns their expert and back.

Dispatch sorts the N*k (token, slot) pairs by destination rank, exchanges the
per-rank counts, moves the token rows with an all-to-all, runs the local
experts as one grouped-GEMM MoE call (every received row has exactly one local
expert), returns the rows with the reverse all-to-all and combines them with
the routing weights at the source, so router gradients flow as in the local
layer.  The reference's EP exchanged only the counts and computed on a zero
buffer, so every MoE layer returned zeros (reference:
distributed/expert_parallel.py:103-137).

This NCCL path needs the split sizes on the host (one small device-to-host copy
per layer) like other all-to-all based MoE implementations.
"""

from __future__ import annotations

from typing import List

import torch
import torch.distributed as dist
import torch.nn as nn

from .. import ops


def _all_to_all(x: torch.Tensor, send: List[int], recv: List[int], group) -> torch.Tensor:
    ws = dist.get_world_size(group)
    out = torch.empty((sum(recv),) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    if dist.get_backend(group) == "nccl":
        dist.all_to_all_single(out, x.contiguous(), recv, send, group=group)
        return out
    # Gloo has no all-to-all: gather every rank's (padded) send buffer instead.
    rank = dist.get_rank(group)
    sizes = torch.tensor([x.shape[0]], dtype=torch.long)
    all_sizes = [torch.zeros(1, dtype=torch.long) for _ in range(ws)]
    dist.all_gather(all_sizes, sizes, group=group)
    cap = int(max(s.item() for s in all_sizes))
    pad = torch.zeros((cap,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    pad[:x.shape[0]] = x
    bufs = [torch.empty_like(pad) for _ in range(ws)]
    dist.all_gather(bufs, pad, group=group)
    splits = torch.tensor(send, dtype=torch.long)
    all_splits = [torch.zeros(ws, dtype=torch.long) for _ in range(ws)]
    dist.all_gather(all_splits, splits, group=group)
    o = 0
    for src in range(ws):
        sp = all_splits[src]
        start = int(sp[:rank].sum())
        n = int(sp[rank])
        out[o:o + n] = bufs[src][start:start + n]
        o += n
    return out


class _AllToAll(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, send, recv, group):
        ctx.send, ctx.recv, ctx.group = send, recv, group
        return _all_to_all(x, send, recv, group)

    @staticmethod
    def backward(ctx, g):
        return _all_to_all(g.contiguous(), ctx.recv, ctx.send, ctx.group), None, None, None


class ExpertParallel:
    """``fused``: use the peer-memory dispatch/combine kernels
    (``parallel.ep_fused``) instead of NCCL all-to-alls.  ``shared`` holds the
    communication buffers common to every MoE layer of the model."""

    def __init__(self, group, num_experts: int, fused: bool = False, shared=None, layer: int = 0):
        self.group = group
        self.ep = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        assert num_experts % self.ep == 0, "num_experts must divide by ep_size"
        self.e_local = num_experts // self.ep
        self.e0 = self.rank * self.e_local
        self.num_experts = num_experts
        self.fused = fused
        self.shared = shared if shared is not None else {}
        self.layer = layer

    def _comm(self, x: torch.Tensor, top_k: int):
        from .ep_fused import EPComm
        N, H = x.shape
        key = (N, H, top_k)
        comm = self.shared.get(key)
        if comm is None:
            comm = self.shared[key] = EPComm(self.group, self.num_experts, H, N, top_k, x.device)
        return comm

    def covers(self, group, x: torch.Tensor) -> bool:
        """True when the fused exchange's counts already span ``group`` (the
        group the load-balancing statistics are summed over)."""
        if not (self.fused and x.is_cuda):
            return False
        mine = dist.get_process_group_ranks(self.group)
        other = dist.get_process_group_ranks(group) if group is not None else list(range(dist.get_world_size()))
        return sorted(mine) == sorted(other)

    def global_stats(self, x: torch.Tensor, counts: torch.Tensor, top_k: int):
        """Global-batch routing statistics from the fused counts exchange: runs
        this layer's layout exchange now (the dispatch reuses it) and sums every
        source's per-expert counts on the device, so the load-balancing loss
        needs no separate all-reduce.  Returns (counts per expert, tokens)."""
        from .ep_fused import ep_layout
        comm = self._comm(x, top_k)
        self._layout = ep_layout(comm, counts)
        tab = comm.counts.view(comm.world, comm.E).float()
        g = tab.sum(0)
        return g, g.sum() / top_k

    def __call__(self, moe, x: torch.Tensor, weights: torch.Tensor, idx: torch.Tensor,
                 counts=None) -> torch.Tensor:
        if self.fused and x.is_cuda:
            from .ep_fused import ep_moe
            comm = self._comm(x, idx.shape[1])
            if counts is None:
                counts = torch.bincount(idx.reshape(-1).long(), minlength=self.num_experts).float()
            layout, self._layout = getattr(self, "_layout", None), None
            return ep_moe(moe, x, weights, idx, counts, comm, self.layer, layout)
        return self._nccl(moe, x, weights, idx)

    def _nccl(self, moe, x: torch.Tensor, weights: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
        N, H = x.shape
        k = idx.shape[1]
        flat = idx.reshape(-1).long()
        dest = torch.div(flat, self.e_local, rounding_mode="floor")
        order = torch.argsort(dest, stable=True)
        send_counts = torch.bincount(dest, minlength=self.ep)
        recv_counts = torch.empty_like(send_counts)
        if dist.get_backend(self.group) == "nccl":
            dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        else:
            recv_counts = _all_to_all(send_counts.view(-1, 1), [1] * self.ep, [1] * self.ep,
                                      self.group).view(-1)
        sc = send_counts.tolist()
        rc = recv_counts.tolist()
        tok = torch.div(order, k, rounding_mode="floor")
        x_send = x[tok]
        e_send = (flat[order] - dest[order] * self.e_local).to(torch.int32)
        x_recv = _AllToAll.apply(x_send, sc, rc, self.group)
        e_recv = _all_to_all(e_send.view(-1, 1), sc, rc, self.group).view(-1)
        R = x_recv.shape[0]
        if R > 0:
            w1 = torch.ones(R, 1, dtype=torch.float32, device=x.device)
            w_gu, w_d = moe.expert_weight_refs(x_recv.dtype)
            y_recv = ops.moe_ffn(x_recv, w1, e_recv.view(R, 1), w_gu, w_d, self.e_local, moe.inter,
                                 None)
        else:
            y_recv = x_recv * 0
        y_send = _AllToAll.apply(y_recv, rc, sc, self.group)
        y_slot = torch.zeros_like(y_send).index_copy(0, order, y_send)
        return (y_slot.view(N, k, H).float() * weights.unsqueeze(-1)).sum(1).to(x.dtype)


def apply_expert_parallel(model: nn.Module, ep_group, fused=None) -> nn.Module:
    """Keep only this rank's experts in every MoE layer and route through EP.

    ``fused`` (default: on CUDA with symmetric memory and 2, 4 or 8 ranks)
    selects the peer-memory dispatch/combine kernels."""
    from ..models.moe import MoELayer
    ws = dist.get_world_size(ep_group)
    r = dist.get_rank(ep_group)
    if fused is None:
        from .peer_dp import symmetric_available
        fused = symmetric_available(ep_group)
    shared: dict = {}
    n_layer = 0
    for m in model.modules():
        if isinstance(m, MoELayer):
            ep = ExpertParallel(ep_group, m.num_experts, fused=bool(fused), shared=shared,
                                layer=n_layer)
            n_layer += 1
            keep = list(range(r * ep.e_local, (r + 1) * ep.e_local))
            m.experts = nn.ModuleList([m.experts[i] for i in keep])
            m.expert_offset = keep[0]
            m.ep = ep
            for p in m.experts.parameters():
                p._ep_local = True
    return model


# Reference-compatible wrapper name (reference: distributed/expert_parallel.py:20)
class ExpertParallelMoE(nn.Module):
    def __init__(self, moe_layer: nn.Module, ep_group=None):
        super().__init__()
        self.moe_layer = moe_layer
        if ep_group is not None and dist.get_world_size(ep_group) > 1:
            r = dist.get_rank(ep_group)
            ep = ExpertParallel(ep_group, moe_layer.num_experts)
            keep = list(range(r * ep.e_local, (r + 1) * ep.e_local))
            moe_layer.experts = nn.ModuleList([moe_layer.experts[i] for i in keep])
            moe_layer.ep = ep

    def forward(self, hidden_states):
        return self.moe_layer(hidden_states)
