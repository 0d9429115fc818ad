"""Context parallelism: the sequence is split over the CP group.

Layout: the sequence is cut into 2*cp equal chunks and rank r holds chunks r
and 2*cp-1-r ("zigzag"), so every rank gets the same amount of causal work.
Tokens keep their global positions (RoPE and the causal mask use them).

Attention: each rank projects q/k/v for its own tokens, all-gathers k and v
(and their positions) over the group -- with GQA the k|v rows are a quarter of
the q rows or less, and over NVSwitch the gather is one collective -- and
attends its queries to every key whose position is not after the query's.  The
backward of the gather is a reduce-scatter of dk/dv.  Gradients of the
replicated parameters are partial sums over the group; ``cp_loss`` scales the
backward by cp so that the engine's gradient average over the (dp x cp) group
yields the data-parallel mean of the full-sequence gradient.

The reference's ring attention (reference: distributed/context_parallel.py:52-136)
is also provided under its name, with a correct source rank per ring step (the
reference receives from rank-1 but masks as if the chunk came from rank+1).
"""

from __future__ import annotations

import math
from typing import Optional

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

from .tensor_parallel import all_gather_dim, reduce_scatter_dim


def zigzag_indices(seq_len: int, cp: int, rank: int, device=None) -> torch.Tensor:
    """Global positions held by ``rank`` (chunks rank and 2cp-1-rank)."""
    if seq_len % (2 * cp):
        raise ValueError(f"seq_len={seq_len} must divide by 2*cp_size={2 * cp}")
    c = seq_len // (2 * cp)
    a = torch.arange(rank * c, (rank + 1) * c, device=device)
    b = torch.arange((2 * cp - 1 - rank) * c, (2 * cp - rank) * c, device=device)
    return torch.cat([a, b])


def split_sequence(hidden_states: torch.Tensor, cp_rank: int, cp_size: int) -> torch.Tensor:
    """Contiguous split along dim 1 (reference API:
    distributed/context_parallel.py:17)."""
    S = hidden_states.shape[1]
    assert S % cp_size == 0, f"seq_len={S} not divisible by cp_size={cp_size}"
    c = S // cp_size
    return hidden_states[:, cp_rank * c:(cp_rank + 1) * c].contiguous()


def gather_sequence(local_hidden: torch.Tensor, cp_group=None) -> torch.Tensor:
    """All-gather contiguous chunks back to the full sequence (reference API:
    distributed/context_parallel.py:38)."""
    if cp_group is None or dist.get_world_size(cp_group) <= 1:
        return local_hidden
    return all_gather_dim(local_hidden, 1, cp_group)


class _GatherKV(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return all_gather_dim(x, 1, group)

    @staticmethod
    def backward(ctx, g):
        return reduce_scatter_dim(g.contiguous(), 1, ctx.group), None


class _CPLoss(torch.autograd.Function):
    """Forward: sum of the per-rank partial losses.  Backward: cp * grad, see
    the module docstring."""

    @staticmethod
    def forward(ctx, part, group):
        ctx.ws = dist.get_world_size(group)
        out = part.clone()
        dist.all_reduce(out, group=group)
        return out

    @staticmethod
    def backward(ctx, g):
        return g * ctx.ws, None


def cp_loss(part: torch.Tensor, group) -> torch.Tensor:
    return _CPLoss.apply(part, group)


def cp_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, pos: torch.Tensor,
                 group, scale: Optional[float] = None) -> torch.Tensor:
    """q [B,Sl,Hq,D], k/v [B,Sl,Hk,D] local; pos [B,Sl] global positions.

    Returns [B,Sl,Hq,D]: causal attention over the whole sequence by position.
    """
    B, Sl, Hq, D = q.shape
    Hk = k.shape[2]
    scale = scale if scale is not None else 1.0 / math.sqrt(D)
    kf = _GatherKV.apply(k, group)
    vf = _GatherKV.apply(v, group)
    pk = all_gather_dim(pos, 1, group)                       # [B, S]
    keep = pk[:, None, :] <= pos[:, :, None]                 # [B, Sl, S]
    g = Hq // Hk
    if g > 1:
        kf = kf.repeat_interleave(g, dim=2)
        vf = vf.repeat_interleave(g, dim=2)
    o = F.scaled_dot_product_attention(q.transpose(1, 2), kf.transpose(1, 2), vf.transpose(1, 2),
                                       attn_mask=keep[:, None], scale=scale)
    return o.transpose(1, 2)


class CPComm:
    """Symmetric buffers and flags of the peer-memory K/V exchange
    (``csrc/cp_comm.cu``): one gathered k|v buffer per attention layer (kept
    for the backward) and two ping-pong dk|dv partial buffers."""

    def __init__(self, group, device):
        from .peer_dp import SymmetricAllocator
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.alloc = SymmetricAllocator(group)
        self.flags = self.alloc(2 * 8, torch.int32, device)
        torch.cuda.synchronize()
        self.p_flags = self.alloc.peer_ptrs(self.flags)
        self.counter = torch.zeros(1, dtype=torch.int32, device=device)
        self.count = 0
        self.seq = [0, 0]
        self.kv = {}
        self.dkv = {}
        dist.barrier(group=group)

    def _buf(self, numel, dtype):
        t = self.alloc(numel, dtype, self.flags.device)
        torch.cuda.synchronize()
        return t, self.alloc.peer_ptrs(t)

    def kv_buf(self, layer, numel):
        key = (layer, numel)
        if key not in self.kv:  # collective: same order on every rank
            self.kv[key] = self._buf(numel, torch.bfloat16)
        return self.kv[key]

    def dkv_buf(self, parity, numel):
        key = (parity, numel)
        if key not in self.dkv:
            self.dkv[key] = self._buf(numel, torch.float32)
        return self.dkv[key]

    def next(self, ch):
        self.seq[ch] += 1
        return self.seq[ch]


class _CPAttnKernelFn(torch.autograd.Function):
    """GPU context-parallel attention on the sm_100a kernels.

    Forward: fused QK-norm + RoPE at the local tokens' global positions, k|v of
    the local tokens gathered over the group into natural position order, then
    ``attn_fwd_cp``: the rank's two zigzag query chunks against the gathered
    keys, causal by position, in one launch.  Backward: ``attn_bwd_cp`` gives
    dq for the local queries and this rank's partial dk|dv for every gathered
    key; the partials are reduce-scattered back to the keys' owners and the
    QK-norm/RoPE backward runs locally.
    """

    @staticmethod
    def forward(ctx, qkv, q_w, k_w, cos, sin, pos, group, Hq, Hk, D, eps, scale, comm, layer):
        from ..ops._ext import ext
        E = ext()
        B, S, W = qkv.shape
        cp = dist.get_world_size(group)
        r = dist.get_rank(group)
        c = S // 2
        Sk = S * cp
        qkv2 = qkv.reshape(B * S, W).contiguous()
        pos1 = pos.reshape(-1).contiguous()
        qk, rstd = E.qknorm_rope_fwd(qkv2, q_w, k_w, cos, sin, pos1, B, S, Hq, Hk, D, float(eps))
        order = torch.cat([zigzag_indices(Sk, cp, q, qkv.device) for q in range(cp)])
        off0, off1 = r * c, (2 * cp - 1 - r) * c
        if comm is not None:
            # every rank stores its rows straight into every rank's gathered buffer;
            # the attention producer waits per key block for the owner's flag
            kvb, kv_ptrs = comm.kv_buf(layer, B * Sk * 2 * Hk * D)
            kv_nat = kvb.view(B * Sk, 2 * Hk * D)
            seq = comm.next(0)
            grid = E.cp_kv_scatter(kv_ptrs, comm.p_flags, comm.rank, qk, qkv2, pos1, B, S, Sk, Hq, Hk, D,
                                   seq, comm.counter, comm.count)
            comm.count += int(grid)
            o, lse = E.attn_fwd_cp(qk, kv_nat, B, S, Sk, Hq, Hk, D, off0, off1, c, float(scale),
                                   comm.flags.data_ptr(), seq, cp)
        else:
            kv_loc = torch.cat([qk[:, Hq * D:], qkv2[:, (Hq + Hk) * D:]], dim=1).view(B, S, 2 * Hk * D)
            kv_all = all_gather_dim(kv_loc.contiguous(), 1, group)      # [B, cp*S] rank-major
            kv_nat = torch.empty_like(kv_all)
            kv_nat[:, order] = kv_all                                   # natural positions
            kv_nat = kv_nat.reshape(B * Sk, 2 * Hk * D).contiguous()
            o, lse = E.attn_fwd_cp(qk, kv_nat, B, S, Sk, Hq, Hk, D, off0, off1, c, float(scale), 0, 0, cp)
        ctx.save_for_backward(qkv2, qk, rstd, kv_nat, o, lse, q_w, k_w, cos, sin, pos1, order)
        ctx.meta = (B, S, cp, Hq, Hk, D, float(scale), off0, off1, c)
        ctx.group, ctx.comm = group, comm
        return o.view(B, S, Hq * D)

    @staticmethod
    def backward(ctx, do):
        from ..ops._ext import ext
        from ..ops.common import grad_buffer
        E = ext()
        qkv2, qk, rstd, kv_nat, o, lse, q_w, k_w, cos, sin, pos, order = ctx.saved_tensors
        B, S, cp, Hq, Hk, D, scale, off0, off1, c = ctx.meta
        do2 = do.reshape(B * S, Hq * D).to(torch.bfloat16).contiguous()
        comm = ctx.comm
        Sk = S * cp
        if comm is not None:
            seq = comm.next(1)
            dkb, dk_ptrs = comm.dkv_buf(seq % 2, B * Sk * 2 * Hk * D)
            dqk, _ = E.attn_bwd_cp(do2, qk, kv_nat, o, lse, B, S, Sk, Hq, Hk, D, off0, off1, c, scale, dkb)
            E.cp_signal(dk_ptrs, comm.p_flags, comm.rank, 1, seq)
            dkv_loc = E.cp_dkv_gather(dk_ptrs, comm.p_flags, comm.rank, pos, B, S, Sk, 2 * Hk * D, seq)
        else:
            dqk, dkv = E.attn_bwd_cp(do2, qk, kv_nat, o, lse, B, S, Sk, Hq, Hk, D, off0, off1, c, scale,
                                     None)
            dkv = dkv.view(B, Sk, 2 * Hk * D)[:, order]                  # back to rank-major
            dkv_loc = reduce_scatter_dim(dkv.contiguous(), 1, ctx.group).reshape(B * S, 2 * Hk * D)
        dqk[:, Hq * D:] = dkv_loc[:, :Hk * D]
        dqkv = torch.empty_like(qkv2)
        dqkv[:, (Hq + Hk) * D:] = dkv_loc[:, Hk * D:].to(dqkv.dtype)
        dqw = grad_buffer(q_w) if (q_w is not None and q_w.requires_grad) else None
        dkw = grad_buffer(k_w) if (k_w is not None and k_w.requires_grad) else None
        E.qknorm_rope_bwd(dqk, qkv2, q_w, k_w, rstd, cos, sin, pos, dqkv, dqw, dkw,
                          B, S, Hq, Hk, D)
        return (dqkv.view(B, S, -1),) + (None,) * 13


_COMMS = {}


def cp_comm(group, device):
    """The peer-memory exchange for ``group`` (None when symmetric memory is
    unavailable: the NCCL all-gather path is used then)."""
    from .peer_dp import symmetric_available
    key = id(group)
    if key not in _COMMS:
        _COMMS[key] = CPComm(group, device) if symmetric_available(group) else None
    return _COMMS[key]


def cp_attention_kernel(qkv, q_w, k_w, cos, sin, pos, group, Hq, Hk, D, eps, scale=None, layer=0):
    """qkv [B, S_local, (Hq+2Hk)*D] of this rank's zigzag tokens at global
    positions ``pos`` -> attention output [B, S_local, Hq*D] (CUDA)."""
    scale = scale if scale is not None else 1.0 / math.sqrt(D)
    comm = cp_comm(group, qkv.device)
    return _CPAttnKernelFn.apply(qkv, q_w, k_w, cos, sin, pos.contiguous(), group, Hq, Hk, D, eps,
                                 scale, comm, layer)


def kernel_usable(S_local: int) -> bool:
    """The CP attention kernels tile query chunks of 256 rows."""
    return torch.cuda.is_available() and S_local % 512 == 0


def apply_context_parallel(model: nn.Module, cp_group, cp_ranks=None,
                           mode: str = "allgather") -> nn.Module:
    """Mark a Qwen3Model (or the LM of a VL model) for context parallelism.
    ``mode``: "allgather" (every rank gathers the group's k|v: one exchange
    per layer, peer-memory kernels on GPUs) or "ring" (k|v blocks passed
    around the group, ``parallel.ring_attention``: two blocks per rank in
    memory, for sequences whose gathered k|v would not fit)."""
    from ..models.attention import Attention
    if mode not in ("allgather", "ring"):
        raise ValueError(f"cp mode {mode!r}: allgather or ring")
    lm = getattr(model, "language_model", model)
    lm.cp_group = cp_group
    for m in lm.modules():
        if isinstance(m, Attention):
            m.cp_group = cp_group
            m.cp_mode = mode
    return model


class RingAttention(nn.Module):
    """Ring attention over contiguous sequence chunks (reference API:
    distributed/context_parallel.py:52).  q/k/v are [B,H,S_local,D]; K/V blocks
    travel one hop per step while the local block is attended; partial results
    are merged with their log-sum-exp.  Differentiable through autograd of the
    per-step math (the p2p exchange itself is treated as constant, as in the
    reference); the model's CP path uses ``cp_attention``."""

    def __init__(self, cp_group=None):
        super().__init__()
        self.cp_group = cp_group
        self.cp_size = dist.get_world_size(cp_group) if cp_group is not None else 1
        self.cp_rank = dist.get_rank(cp_group) if cp_group is not None else 0

    def forward(self, q, k, v, causal: bool = True):
        if self.cp_size <= 1:
            return F.scaled_dot_product_attention(q, k, v, is_causal=causal)
        B, H, S, D = q.shape
        scale = 1.0 / math.sqrt(D)
        ranks = dist.get_process_group_ranks(self.cp_group)
        nxt = ranks[(self.cp_rank + 1) % self.cp_size]
        prv = ranks[(self.cp_rank - 1) % self.cp_size]
        out = torch.zeros(B, H, S, D, dtype=torch.float32, device=q.device)
        lse = torch.full((B, H, S, 1), float("-inf"), device=q.device)
        kc, vc = k.contiguous(), v.contiguous()
        for step in range(self.cp_size):
            src = (self.cp_rank - step) % self.cp_size   # owner of the block held now
            if step < self.cp_size - 1:
                kr, vr = torch.empty_like(kc), torch.empty_like(vc)
                ops = [dist.P2POp(dist.isend, kc, nxt, self.cp_group),
                       dist.P2POp(dist.isend, vc, nxt, self.cp_group),
                       dist.P2POp(dist.irecv, kr, prv, self.cp_group),
                       dist.P2POp(dist.irecv, vr, prv, self.cp_group)]
                reqs = dist.batch_isend_irecv(ops)
            if not (causal and src > self.cp_rank):
                s = torch.matmul(q.float(), kc.float().transpose(-2, -1)) * scale
                if causal and src == self.cp_rank:
                    m = torch.triu(torch.ones(S, S, dtype=torch.bool, device=q.device), 1)
                    s = s.masked_fill(m, float("-inf"))
                blk_lse = torch.logsumexp(s, -1, keepdim=True)
                blk = torch.matmul(torch.exp(s - blk_lse), vc.float())
                new = torch.logaddexp(lse, blk_lse)
                out = out * torch.exp(lse - new) + blk * torch.exp(blk_lse - new)
                lse = new
            if step < self.cp_size - 1:
                for r in reqs:
                    r.wait()
                kc, vc = kr, vr
        return out.to(q.dtype)
