"""Expert parallelism with dispatch and combine as this library's own kernels
over NVLink peer memory (``csrc/ep_comm.cu``).

Forward of one MoE layer on rank r (experts [r*El, (r+1)*El)):

1. ``ep_layout``: every rank publishes its per-expert routing counts into every
   rank's count table; each rank then knows the full [ranks x experts] matrix
   and computes, on the device, where each of its (token, slot) pairs lands in
   the owner's receive buffer (128-row aligned segment per expert, sources in
   rank order) and its own segment offsets for the grouped GEMMs.
2. ``ep_dispatch``: each pair's token row is stored straight into the owner's
   receive buffer (P2P stores; the permutation and the all-to-all are one
   pass); padding rows of the own buffer are zeroed.
3. The grouped gate|up GEMM (tcgen05) consumes the receive buffer directly:
   before loading a tile of an expert segment its TMA producer waits for the
   dispatch flags of the source ranks whose rows the tile covers, so tiles
   start as their rows land; SwiGLU and the grouped down GEMM follow.
4. ``ep_combine``: each source pulls its pairs' output rows from the owners
   (P2P loads) and forms the weighted top-k sum.

The backward pushes the weighted output gradient to the owners, runs the
grouped backward GEMMs there and pulls the input gradient back.  No step
synchronises with the host; the receive capacity is fixed when the buffers
are created (``capacity_factor`` x the average rows per rank, or the exact
worst case when that is smaller) and overflowing pairs are dropped with an
error code instead of being written out of bounds.
"""

from __future__ import annotations

import math
from typing import Dict, List, Tuple

import torch
import torch.distributed as dist

from ..ops._ext import ext
from .peer_dp import SymmetricAllocator

CH_COUNTS, CH_DISPATCH, CH_OUT, CH_DOUT, CH_DX = 0, 1, 2, 3, 4


class EPComm:
    def __init__(self, group, num_experts: int, hidden: int, tokens: int, top_k: int,
                 device: torch.device, capacity_factor: float = 2.0):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.E = num_experts
        self.El = num_experts // self.world
        self.H = hidden
        self.N = tokens
        worst = self.world * tokens * top_k
        avg = tokens * top_k
        self.cap = min(worst, int(math.ceil(capacity_factor * avg))) + self.El * 128
        self.cap = (self.cap + 127) // 128 * 128
        self.alloc = SymmetricAllocator(group)
        self.flags = self.alloc(8 * 8, torch.int32, device)
        self.counts = self.alloc(self.world * num_experts, torch.int32, device)
        torch.cuda.synchronize()
        self.p_flags = self.alloc.peer_ptrs(self.flags)
        self.p_counts = self.alloc.peer_ptrs(self.counts)
        self.y_out = self._buf()
        self.dy_recv = self._buf()
        # two input-gradient staging buffers, by MoE-layer parity: an owner
        # whose dgrad waits for no rows of some source (that source routed
        # nothing to it in this layer) could otherwise overwrite the buffer
        # while that source still pulls the previous layer's rows from it
        self.dx_recv = [self._buf(), self._buf()]
        self.recv: Dict[int, Tuple[torch.Tensor, List[int]]] = {}
        self.counter = torch.zeros(1, dtype=torch.int32, device=device)
        self.count = 0
        self.seq = [0] * 8
        dist.barrier(group=group)

    def _buf(self) -> Tuple[torch.Tensor, List[int]]:
        t = self.alloc(self.cap * self.H, torch.bfloat16, self.flags.device).view(self.cap, self.H)
        torch.cuda.synchronize()
        return t, self.alloc.peer_ptrs(t)

    def recv_buf(self, layer: int) -> Tuple[torch.Tensor, List[int]]:
        if layer not in self.recv:
            self.recv[layer] = self._buf()  # collective: same order on every rank
        return self.recv[layer]

    def next(self, ch: int) -> int:
        self.seq[ch] += 1
        return self.seq[ch]

    def ep_wait_args(self, ch: int, seq: int, counts: torch.Tensor) -> dict:
        """Arguments that make a grouped GEMM wait per tile for channel
        ``ch``'s flags (this rank's slots, one per source) to reach ``seq``;
        ``counts`` is the [ranks x experts] table of the layer whose rows
        arrive (the live table belongs to the most recent layout)."""
        return dict(ep_counts=counts.data_ptr(), ep_flags=self.flags.data_ptr() + ch * 8 * 4,
                    ep_seq=seq, ep_world=self.world, ep_E=self.E, ep_expert0=self.rank * self.El)

    def advance(self, grid: int) -> int:
        before = self.count
        self.count += int(grid)
        return before


def _grad_view(wref, shape):
    if wref.grad is None:
        raise RuntimeError("expert weights must live in a FlatParamStore on GPU")
    return wref.grad.view(shape)


def ep_layout(comm: EPComm, counts: torch.Tensor):
    """Counts exchange + receive layout of one MoE layer (``ep_layout``): every
    rank's per-expert counts land in every rank's table; returns
    (dest_base [E], seg_off [El+1], seg_used [El])."""
    E = ext()
    dev = counts.device
    dest_base = torch.empty(comm.E, dtype=torch.int32, device=dev)
    seg_off = torch.empty(comm.El + 1, dtype=torch.int32, device=dev)
    seg_used = torch.empty(comm.El, dtype=torch.int32, device=dev)
    s0 = comm.next(CH_COUNTS)
    E.ep_layout(comm.p_flags, comm.p_counts, comm.rank, counts.float().contiguous(), comm.E, comm.El, s0,
                dest_base, seg_off, seg_used, comm.cap)
    return dest_base, seg_off, seg_used


class _EPMoE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weights, idx, counts, w_gu, w_d, comm: EPComm, layer: int, inter: int, layout,
                *anchors):
        E = ext()
        N, H = x.shape
        K = idx.shape[1]
        dev = x.device
        El = comm.El
        idx = idx.to(torch.int32).contiguous()
        x = x.contiguous()
        # the layout may already have run (global load-balancing statistics)
        dest_base, seg_off, seg_used = layout if layout is not None else ep_layout(comm, counts)
        # this layer's [ranks x experts] counts: the shared table is rewritten
        # by every later layer's layout, and the backward's row waits need
        # this layer's (copied before any peer can start the next layout:
        # a peer's next layout follows its combine, which waits for this
        # rank's expert outputs, which follow this copy in stream order)
        cnt = comm.counts.clone()
        slot_of, loc_off, _ = E.moe_plan(idx, comm.E, -1, 1)  # pad 1: unpadded order
        recv, recv_ptrs = comm.recv_buf(layer)
        dest_row = torch.empty(N, K, dtype=torch.int32, device=dev)
        s1 = comm.next(CH_DISPATCH)
        before = comm.count
        grid = E.ep_dispatch(comm.p_flags, comm.p_counts, recv_ptrs, comm.rank, x, idx, slot_of, loc_off,
                             dest_base, seg_off, seg_used, dest_row, El, comm.cap, s1, comm.counter, before)
        comm.advance(grid)
        Wgu = w_gu.compute.view(El, 2 * inter, H)
        Wd = w_d.compute.view(El, H, inter)
        # the gate|up GEMM consumes the receive buffer as rows land: its TMA
        # producer waits, per tile, for the dispatch flags of the sources
        # whose rows the tile covers (no separate wait for all sources)
        gu = E.grouped_gemm_nt(recv, Wgu, seg_off, **comm.ep_wait_args(CH_DISPATCH, s1, cnt))
        h = E.swiglu_fwd(gu)
        y = E.grouped_gemm_nt(h, Wd, seg_off)
        yo, yo_ptrs = comm.y_out
        yo.copy_(y)
        s2 = comm.next(CH_OUT)
        E.ep_signal(comm.p_flags, comm.p_counts, comm.rank, CH_OUT, s2)
        out = torch.empty(N, H, dtype=x.dtype, device=dev)
        y_pulled = torch.empty(N * K, H, dtype=x.dtype, device=dev)
        w32 = weights.float().contiguous()
        E.ep_combine(comm.p_flags, comm.p_counts, yo_ptrs, comm.rank, idx, dest_row, w32, out, y_pulled,
                     El, s2)
        ctx.save_for_backward(idx, dest_row, w32, y_pulled, seg_off, recv, gu, h, cnt)
        ctx.comm, ctx.w, ctx.meta = comm, (w_gu, w_d), (El, inter, H, len(w_gu.anchors) + len(w_d.anchors))
        ctx.layer = layer
        return out

    @staticmethod
    def backward(ctx, dout):
        idx, dest_row, w32, y_pulled, seg_off, recv, gu, h, cnt = ctx.saved_tensors
        comm: EPComm = ctx.comm
        w_gu, w_d = ctx.w
        El, inter, H, n_anchor = ctx.meta
        E = ext()
        N, K = idx.shape
        dout = dout.contiguous().to(torch.bfloat16)
        dw = torch.empty(N, K, dtype=torch.float32, device=dout.device)
        dyr, dyr_ptrs = comm.dy_recv
        s3 = comm.next(CH_DOUT)
        before = comm.count
        grid = E.ep_combine_bwd(comm.p_flags, comm.p_counts, dyr_ptrs, comm.rank, idx, dest_row, w32, dout,
                                y_pulled, dw, El, s3, comm.counter, before)
        comm.advance(grid)
        Wgu = w_gu.compute.view(El, 2 * inter, H)
        Wd = w_d.compute.view(El, H, inter)
        # the down-projection dgrad consumes the pushed output gradients as
        # they land (per-tile waits on the sources' flags); the weight
        # gradient runs after it in stream order, on complete data
        dh = E.grouped_gemm_nn(dyr, Wd, seg_off, **comm.ep_wait_args(CH_DOUT, s3, cnt))
        if w_d.requires_grad:
            E.grouped_gemm_tn_acc(dyr, h, _grad_view(w_d, (El, H, inter)), seg_off)
        dgu = E.swiglu_bwd(dh, gu)
        if w_gu.requires_grad:
            E.grouped_gemm_tn_acc(dgu, recv, _grad_view(w_gu, (El, 2 * inter, H)), seg_off)
        dxr = E.grouped_gemm_nn(dgu, Wgu, seg_off)
        dxo, dxo_ptrs = comm.dx_recv[ctx.layer % 2]
        dxo.copy_(dxr)
        s4 = comm.next(CH_DX)
        E.ep_signal(comm.p_flags, comm.p_counts, comm.rank, CH_DX, s4)
        dx = torch.empty(N, H, dtype=torch.bfloat16, device=dout.device)
        E.ep_dispatch_bwd(comm.p_flags, comm.p_counts, dxo_ptrs, comm.rank, idx, dest_row, dx, El, s4)
        return (dx, dw, None, None, None, None, None, None, None, None) + (None,) * n_anchor


def ep_moe(moe, x, weights, idx, counts, comm: EPComm, layer: int, layout=None) -> torch.Tensor:
    w_gu, w_d = moe.expert_weight_refs(x.dtype)
    return _EPMoE.apply(x, weights, idx, counts, w_gu, w_d, comm, layer, moe.inter, layout,
                        *w_gu.anchors, *w_d.anchors)
