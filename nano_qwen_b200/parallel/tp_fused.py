"""Tensor + sequence parallelism with the collectives fused into the kernels
(GPU, NVLink peer memory).

The sequence-parallel residual stream is split over the flattened tokens: rank
r holds rows [r*R, (r+1)*R) of the [B*S, H] stream, so the rank-major
full-sequence buffer *is* the token order attention expects.  Per block:

    norm_1:  h = resid + sum(partials of the previous down_proj)   (reduce-scatter's sum)
             y = rmsnorm(h) -> stored into every rank's x_full      (all-gather)
    q|k|v:   GEMM over x_full; its TMA producer waits per row tile for the
             owner's all-gather flag
    attention on the rank's heads over the full sequence
    o_proj:  GEMM whose epilogue stores row tiles into their owner's partial
             buffer (reduce-scatter without a separate pass)
    norm_2, gate|up, SwiGLU, down_proj: the same pattern

Backward mirrors it (dgrad GEMMs of the column-parallel layers reduce-scatter
into the norms' backward, the norms' backward all-gathers the residual
gradient that the row-parallel layers' dgrad/wgrad GEMMs read).  Kernels:
``csrc/tp_comm.cu`` (norms) and the AG/RS variants of ``csrc/gemm.cu``.

Buffers live in symmetric memory: one x_full per (layer, norm) (kept for the
weight-gradient GEMMs), and ping-pong partial / gradient buffers.  Flags are
monotonic sequence numbers per channel, identical on every rank because every
rank issues the same sequence of operations.
"""

from __future__ import annotations

from typing import Dict, List, Tuple

import torch
import torch.distributed as dist

from .. import ops
from ..ops._ext import ext
from .peer_dp import SymmetricAllocator

AG_FWD, RS_FWD, AG_BWD, RS_BWD = 0, 1, 2, 3


class TPComm:
    def __init__(self, group, rows: int, hidden: int, device: torch.device):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if rows % 128:
            raise ValueError("fused TP needs tokens per rank divisible by 128")
        self.R, self.H = rows, hidden
        self.alloc = SymmetricAllocator(group)
        self.flags = self.alloc(4 * 8, torch.int32, device)
        self.counter = torch.zeros(1, dtype=torch.int32, device=device)
        self.count = 0
        self.seq = [0, 0, 0, 0]
        torch.cuda.synchronize()
        self.p_flags = self.alloc.peer_ptrs(self.flags)
        W, R, H = self.world, rows, hidden
        self.parts_fwd = [self._buf((W, R, H)) for _ in range(2)]
        self.parts_bwd = [self._buf((W, R, H)) for _ in range(2)]
        self.dy_full = [self._buf((W * R, H)) for _ in range(2)]
        self.x_full: Dict[Tuple[int, int], Tuple[torch.Tensor, List[int]]] = {}
        dist.barrier(group=group)

    def _buf(self, shape) -> Tuple[torch.Tensor, List[int]]:
        n = 1
        for s in shape:
            n *= s
        t = self.alloc(n, torch.bfloat16, self.flags.device).view(*shape)
        torch.cuda.synchronize()
        return t, self.alloc.peer_ptrs(t)

    def xbuf(self, key) -> Tuple[torch.Tensor, List[int]]:
        if key not in self.x_full:
            # collective: every rank creates the same keys in the same order
            self.x_full[key] = self._buf((self.world * self.R, self.H))
        return self.x_full[key]

    def next_seq(self, ch: int) -> int:
        self.seq[ch] += 1
        return self.seq[ch]

    def flag_ptr(self, ch: int) -> int:
        return self.flags.data_ptr() + ch * 8 * 4

    def ag_targets(self, ptrs: List[int]) -> List[int]:
        """Addresses of this rank's rows in every rank's full buffer."""
        off = self.rank * self.R * self.H * 2
        return [p + off for p in ptrs]

    def part_targets(self, ptrs: List[int]) -> List[int]:
        """Addresses of plane [src = this rank] of every rank's partial buffer."""
        off = self.rank * self.R * self.H * 2
        return [p + off for p in ptrs]

    def advance(self, grid: int) -> int:
        before = self.count
        self.count += int(grid)
        return before


class _NormAG(torch.autograd.Function):
    """resid (+delta) (+partials) -> RMSNorm; the output rows are all-gathered
    into ``x_full`` (or kept local when ``ag`` is False)."""

    @staticmethod
    def forward(ctx, resid, delta, dummy, w, comm: TPComm, key, ag: bool, eps: float,
                parts_idx: int, wait_seq: int):
        ctx.set_materialize_grads(False)
        E = ext()
        R, H = comm.R, comm.H
        h = torch.empty(R, H, dtype=torch.float32, device=resid.device)
        y = torch.empty(R, H, dtype=torch.bfloat16, device=resid.device)
        rstd = torch.empty(R, dtype=torch.float32, device=resid.device)
        parts = comm.parts_fwd[parts_idx][0] if parts_idx >= 0 else None
        targets: List[int] = []
        sig_seq = 0
        if ag:
            xf, ptrs = comm.xbuf(key)
            targets = comm.ag_targets(ptrs)
            sig_seq = comm.next_seq(AG_FWD)
        before = comm.count
        grid = E.tp_norm_fwd(resid.reshape(R, H), delta.reshape(R, H) if delta is not None else None,
                             parts, w, h, y, rstd, eps, targets, comm.flags, comm.p_flags, comm.rank,
                             RS_FWD if parts is not None else -1, wait_seq,
                             AG_FWD if ag else -1, sig_seq, comm.counter, before)
        if ag:
            comm.advance(grid)
        ctx.save_for_backward(h, w, rstd)
        ctx.comm, ctx.eps, ctx.ag = comm, eps, ag
        ctx.has_delta = delta is not None
        ctx.has_parts = parts is not None
        out_x = comm.xbuf(key)[0] if ag else y
        return h, out_x

    @staticmethod
    def backward(ctx, dh, dx_in):
        h, w, rstd = ctx.saved_tensors
        comm: TPComm = ctx.comm
        E = ext()
        R, H = comm.R, comm.H
        dx = torch.empty(R, H, dtype=torch.float32, device=h.device)
        dxb = torch.empty(R, H, dtype=torch.bfloat16, device=h.device)
        dw = ops.common.grad_buffer(w) if w.requires_grad else None
        dy_local = None
        dy_parts = None
        wait_seq = 0
        if ctx.ag:
            # gradient of the all-gathered output: tp partials written by the
            # column-parallel dgrad GEMMs of every rank
            wait_seq = comm.seq[RS_BWD]
            dy_parts = comm.parts_bwd[wait_seq % 2][0]
        elif dx_in is not None:
            dy_local = dx_in.reshape(R, H).to(torch.bfloat16).contiguous()
        targets: List[int] = []
        sig_seq = 0
        need_ag = ctx.has_parts  # the row-parallel op before this norm reads the full gradient
        if need_ag:
            sig_seq = comm.next_seq(AG_BWD)
            buf, ptrs = comm.dy_full[sig_seq % 2]
            targets = comm.ag_targets(ptrs)
        before = comm.count
        grid = E.tp_norm_bwd(dy_local, dy_parts, dh.reshape(R, H).contiguous() if dh is not None else None,
                             h, w, rstd, dx, dxb, dw, targets, comm.flags, comm.p_flags, comm.rank,
                             RS_BWD if dy_parts is not None else -1, wait_seq,
                             AG_BWD if need_ag else -1, sig_seq, comm.counter, before)
        if need_ag:
            comm.advance(grid)
        d_resid = dx
        d_delta = dxb if ctx.has_delta else None
        d_dummy = torch.zeros(0, device=h.device) if ctx.has_parts else None
        return d_resid, d_delta, d_dummy, None, None, None, None, None, None, None


class _ColLinear(torch.autograd.Function):
    """Column-parallel GEMM over the all-gathered x_full."""

    @staticmethod
    def forward(ctx, x_full, ag_seq: int, wref, comm: TPComm, *anchors):
        E = ext()
        y = E.gemm_ag(x_full, wref.compute, False, comm.flag_ptr(AG_FWD), ag_seq, comm.R)
        ctx.wref, ctx.comm = wref, comm
        ctx.save_for_backward(x_full)
        return y

    @staticmethod
    def backward(ctx, dy):
        (x_full,) = ctx.saved_tensors
        comm: TPComm = ctx.comm
        wref = ctx.wref
        E = ext()
        dy = dy.contiguous()
        seq = comm.next_seq(RS_BWD)
        buf, ptrs = comm.parts_bwd[seq % 2]
        before = comm.count
        grid = E.gemm_rs(dy, wref.compute, True, comm.part_targets(ptrs), comm.R, comm.counter, before,
                         comm.p_flags, RS_BWD * 8 + comm.rank, seq)
        comm.advance(grid)
        if wref.requires_grad:
            E.gemm_tn_acc(dy, x_full, wref.grad)
        return (None, None, None, None) + (None,) * len(wref.anchors)


class _RowLinear(torch.autograd.Function):
    """Row-parallel GEMM whose row tiles go to their owners' partial buffers;
    returns an empty tensor that carries the dependency to the next norm."""

    @staticmethod
    def forward(ctx, x, wref, comm: TPComm, *anchors):
        E = ext()
        x = x.contiguous()
        seq = comm.next_seq(RS_FWD)
        buf, ptrs = comm.parts_fwd[seq % 2]
        before = comm.count
        grid = E.gemm_rs(x, wref.compute, False, comm.part_targets(ptrs), comm.R, comm.counter, before,
                         comm.p_flags, RS_FWD * 8 + comm.rank, seq)
        comm.advance(grid)
        ctx.wref, ctx.comm = wref, comm
        ctx.save_for_backward(x)
        ctx.seq = seq
        dummy = torch.empty(0, device=x.device)
        return dummy

    @staticmethod
    def backward(ctx, _):
        (x,) = ctx.saved_tensors
        comm: TPComm = ctx.comm
        wref = ctx.wref
        E = ext()
        seq = comm.seq[AG_BWD]
        dy_full, _ = comm.dy_full[seq % 2]
        dx = E.gemm_ag(dy_full, wref.compute, True, comm.flag_ptr(AG_BWD), seq, comm.R)
        if wref.requires_grad:
            E.gemm_tn_acc(dy_full, x, wref.grad)
        return (dx, None, None) + (None,) * len(wref.anchors)


def parts_index(comm: TPComm) -> Tuple[int, int]:
    """(ping-pong index, sequence) of the partials written by the latest row-parallel GEMM."""
    s = comm.seq[RS_FWD]
    return s % 2, s


def block_forward(blk, resid, dummy, comm: TPComm, layer: int, B: int, S: int):
    """One transformer block under fused TP+SP.  resid [R, H] fp32 shard;
    ``dummy`` is the previous row-parallel GEMM's output (None before layer 0)."""
    att, ff = blk.attention, blk.feed_forward
    cfg = blk.config
    eps = cfg.rms_norm_eps
    dt = torch.bfloat16
    pidx, pseq = parts_index(comm) if dummy is not None else (-1, 0)
    h, x_full = _NormAG.apply(resid, None, dummy, blk.input_layernorm.weight, comm, (layer, 0),
                              True, eps, pidx, pseq)
    agseq = comm.seq[AG_FWD]
    wq = ops.weight_ref([att.q_proj.weight, att.k_proj.weight, att.v_proj.weight], dt)
    qkv = _ColLinear.apply(x_full, agseq, wq, comm, *wq.anchors)
    Hq, Hk = att._heads()
    D = att.head_dim
    qw = att.q_norm.weight if att.qk_norm else None
    kw = att.k_norm.weight if att.qk_norm else None
    o = ops.attention_core(qkv.view(B, S, -1), qw, kw, att.rotary_emb.cos_cached,
                           att.rotary_emb.sin_cached, None, Hq, Hk, D, eps, causal=True)
    wo = ops.weight_ref([att.o_proj.weight], dt)
    d1 = _RowLinear.apply(o.view(B * S, -1), wo, comm, *wo.anchors)
    pidx, pseq = parts_index(comm)
    h2, x2_full = _NormAG.apply(h, None, d1, blk.post_attention_layernorm.weight, comm,
                                (layer, 1), True, eps, pidx, pseq)
    agseq2 = comm.seq[AG_FWD]
    wgu = ops.weight_ref([ff.gate_proj.weight, ff.up_proj.weight], dt)
    gu = _ColLinear.apply(x2_full, agseq2, wgu, comm, *wgu.anchors)
    a = ops.swiglu_packed(gu)
    wd = ops.weight_ref([ff.down_proj.weight], dt)
    d2 = _RowLinear.apply(a, wd, comm, *wd.anchors)
    return h2, d2


def final_norm(resid, dummy, w, comm: TPComm, eps: float):
    pidx, pseq = parts_index(comm)
    h, y = _NormAG.apply(resid, None, dummy, w, comm, None, False, eps, pidx, pseq)
    return y


def usable(model) -> bool:
    """Fused TP applies to dense Qwen3 blocks on CUDA with symmetric memory."""
    lm = getattr(model, "language_model", model)
    return torch.cuda.is_available() and not any(lm.config.layer_is_moe(i)
                                                 for i in range(lm.config.num_hidden_layers))
