"""Ring schedule for context-parallel attention (memory bounded by two K/V
blocks per rank instead of the whole sequence).

Layout: the zigzag split of ``parallel.context_parallel`` (the sequence in
2*cp chunks of c tokens, rank r holding chunks r and 2cp-1-r, positions
global), so every rank has the same causal work at every ring step.

Forward, per attention layer: the rank's k|v block (its two chunks) travels
around the ring (send to rank r+1, receive from r-1, the transfer of step s+1
overlapping the attention of step s).  At each step the two local query
chunks meet the two held key chunks; a (query chunk, key chunk) pair is
fully visible (key chunk earlier), causal (same chunk) or invisible (key chunk
later), so each pair is one plain flash-attention call, and the partial
outputs are merged with their log-sum-exp.

Backward: the k|v blocks travel the ring again, each with an fp32 dk|dv
accumulator; a rank adds the gradient of the held block from its queries
(computed with the merged output and log-sum-exp, so each pair's softmax
gradient is the global one) and passes block and accumulator on.  After cp
steps every accumulator is back at its owner.

The pair attention runs on the sm_100a flash kernels for CUDA tensors
(``KernelPair``: ``attn_fwd`` / ``attn_bwd`` on a q chunk and a k|v chunk laid
out as one self-attention call) and on an fp32 statement of attention
otherwise (``TorchPair``).  Exchanges are torch.distributed point-to-point
operations (NCCL on GPUs, Gloo in the CPU tests).

The reference's ring (reference: distributed/context_parallel.py:52-140)
treats the exchanged blocks as constants (no key/value gradient for other
ranks' blocks) and is never wired into its model; this one is the model's
context-parallel attention when ``cp_mode="ring"``.
"""

from __future__ import annotations

import math
from typing import List, Optional, Tuple

import torch
import torch.distributed as dist


def ring_chunks(cp: int, rank: int) -> Tuple[int, int]:
    """Chunk indices (of 2*cp) held by ``rank`` in the zigzag layout."""
    return rank, 2 * cp - 1 - rank


def pair_relation(q_chunk: int, k_chunk: int) -> Optional[bool]:
    """None: no key visible; False: every key visible; True: causal diagonal."""
    if k_chunk > q_chunk:
        return None
    return k_chunk == q_chunk


class TorchPair:
    """fp32 attention of one query chunk [B, c, Hq, D] against one key/value
    chunk [B, c, Hk, D] (grouped-query heads)."""

    @staticmethod
    def _scores(q, k, causal, scale):
        B, c, Hq, D = q.shape
        g = Hq // k.shape[2]
        qf = q.float().transpose(1, 2)                                   # [B, Hq, c, D]
        kf = k.float().transpose(1, 2).repeat_interleave(g, dim=1)       # [B, Hq, c, D]
        s = torch.matmul(qf, kf.transpose(-1, -2)) * scale
        if causal:
            m = torch.ones(c, c, dtype=torch.bool, device=q.device).triu(1)
            s = s.masked_fill(m, float("-inf"))
        return s, qf, kf

    def fwd(self, q, k, v, causal: bool, scale: float):
        g = q.shape[2] // k.shape[2]
        s, _, _ = self._scores(q, k, causal, scale)
        lse = torch.logsumexp(s, -1)                                     # [B, Hq, c]
        vf = v.float().transpose(1, 2).repeat_interleave(g, dim=1)
        o = torch.matmul(torch.exp(s - lse[..., None]), vf)               # [B, Hq, c, D]
        return o.transpose(1, 2), lse

    def bwd(self, do, q, k, v, o, lse, causal: bool, scale: float):
        B, c, Hq, D = q.shape
        Hk = k.shape[2]
        g = Hq // Hk
        s, qf, kf = self._scores(q, k, causal, scale)
        p = torch.exp(s - lse[..., None])
        vf = v.float().transpose(1, 2).repeat_interleave(g, dim=1)
        dof = do.float().transpose(1, 2)
        of = o.float().transpose(1, 2)
        dv = torch.matmul(p.transpose(-1, -2), dof)
        dp = torch.matmul(dof, vf.transpose(-1, -2))
        delta = (dof * of).sum(-1, keepdim=True)
        ds = p * (dp - delta)
        dq = torch.matmul(ds, kf) * scale
        dk = torch.matmul(ds.transpose(-1, -2), qf) * scale
        dk = dk.view(B, Hk, g, c, D).sum(2)
        dv = dv.view(B, Hk, g, c, D).sum(2)
        return dq.transpose(1, 2), dk.transpose(1, 2), dv.transpose(1, 2)


class KernelPair:
    """The same pair on the flash-attention kernels: the query chunk's rows
    and the key/value chunk's rows form one [B*c] self-attention layout
    (q | k | v per row), so ``attn_fwd`` / ``attn_bwd`` run unchanged, full or
    causal."""

    @staticmethod
    def _layout(q, k, v):
        B, c, Hq, D = q.shape
        Hk = k.shape[2]
        qk = torch.cat([q.reshape(B * c, Hq * D), k.reshape(B * c, Hk * D)], 1).to(torch.bfloat16)
        qkv = torch.cat([qk, v.reshape(B * c, Hk * D).to(torch.bfloat16)], 1).contiguous()
        return qk.contiguous(), qkv

    def fwd(self, q, k, v, causal: bool, scale: float):
        from ..ops._ext import ext
        B, c, Hq, D = q.shape
        qk, qkv = self._layout(q, k, v)
        o, lse = ext().attn_fwd(qk, qkv, B, c, Hq, k.shape[2], D, bool(causal), float(scale))
        return o.view(B, c, Hq, D).float(), lse

    def bwd(self, do, q, k, v, o, lse, causal: bool, scale: float):
        from ..ops._ext import ext
        B, c, Hq, D = q.shape
        Hk = k.shape[2]
        qk, qkv = self._layout(q, k, v)
        do2 = do.reshape(B * c, Hq * D).to(torch.bfloat16).contiguous()
        o2 = o.reshape(B * c, Hq * D).to(torch.bfloat16).contiguous()
        dqkv = torch.empty_like(qkv)
        dqk = ext().attn_bwd(do2, qk, qkv, o2, lse.contiguous(), dqkv, B, c, Hq, Hk, D, bool(causal),
                             float(scale))
        dq = dqk[:, :Hq * D].reshape(B, c, Hq, D)
        dk = dqk[:, Hq * D:].reshape(B, c, Hk, D)
        dv = dqkv[:, (Hq + Hk) * D:].float().reshape(B, c, Hk, D)
        return dq, dk, dv


def _exchange(send: List[torch.Tensor], recv: List[torch.Tensor], group):
    """Send to the next rank of the ring, receive from the previous one."""
    ws, r = dist.get_world_size(group), dist.get_rank(group)
    ranks = dist.get_process_group_ranks(group)
    nxt, prv = ranks[(r + 1) % ws], ranks[(r - 1) % ws]
    ops = [dist.P2POp(dist.isend, t, nxt, group) for t in send]
    ops += [dist.P2POp(dist.irecv, t, prv, group) for t in recv]
    return dist.batch_isend_irecv(ops)


def _merge(o_acc, lse_acc, o_p, lse_p):
    """Combine two partial softmax results (o [B, c, H, D], lse [B, H, c])."""
    new = torch.logaddexp(lse_acc, lse_p)
    a = torch.exp(lse_acc - new).transpose(1, 2)[..., None]
    b = torch.exp(lse_p - new).transpose(1, 2)[..., None]
    o_acc.mul_(a).add_(o_p * b)
    lse_acc.copy_(new)


class _RingFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, group, scale, pair):
        B, S, Hq, D = q.shape
        Hk = k.shape[2]
        cp, r = dist.get_world_size(group), dist.get_rank(group)
        c = S // 2
        mine = ring_chunks(cp, r)
        kv = torch.stack([k, v], 2).contiguous()                 # [B, S, 2, Hk, D]
        o = torch.zeros(B, S, Hq, D, dtype=torch.float32, device=q.device)
        lse = torch.full((B, Hq, S), float("-inf"), dtype=torch.float32, device=q.device)
        cur = kv
        for s in range(cp):
            src = (r - s) % cp
            reqs, nxt = None, None
            if s < cp - 1:
                nxt = torch.empty_like(cur)
                reqs = _exchange([cur], [nxt], group)
            for qi, qc in enumerate(mine):
                for kj, kc in enumerate(ring_chunks(cp, src)):
                    rel = pair_relation(qc, kc)
                    if rel is None:
                        continue
                    qs, ks = slice(qi * c, (qi + 1) * c), slice(kj * c, (kj + 1) * c)
                    o_p, lse_p = pair.fwd(q[:, qs], cur[:, ks, 0], cur[:, ks, 1], rel, scale)
                    _merge(o[:, qs], lse[:, :, qs], o_p, lse_p)
            if reqs is not None:
                for rq in reqs:
                    rq.wait()
                cur = nxt
        out = o.to(q.dtype)
        ctx.save_for_backward(q, kv, out, lse)
        ctx.group, ctx.scale, ctx.pair = group, scale, pair
        return out

    @staticmethod
    def backward(ctx, do):
        q, kv, o, lse = ctx.saved_tensors
        group, scale, pair = ctx.group, ctx.scale, ctx.pair
        B, S, Hq, D = q.shape
        cp, r = dist.get_world_size(group), dist.get_rank(group)
        c = S // 2
        mine = ring_chunks(cp, r)
        dq = torch.zeros(B, S, Hq, D, dtype=torch.float32, device=q.device)
        cur = kv
        acc = torch.zeros(kv.shape, dtype=torch.float32, device=q.device)
        for s in range(cp):
            src = (r - s) % cp
            reqs, nxt = None, None
            if s < cp - 1:   # the next block's transfer overlaps this step's math
                nxt = torch.empty_like(cur)
                reqs = _exchange([cur], [nxt], group)
            for qi, qc in enumerate(mine):
                for kj, kc in enumerate(ring_chunks(cp, src)):
                    rel = pair_relation(qc, kc)
                    if rel is None:
                        continue
                    qs, ks = slice(qi * c, (qi + 1) * c), slice(kj * c, (kj + 1) * c)
                    dq_p, dk_p, dv_p = pair.bwd(do[:, qs], q[:, qs], cur[:, ks, 0], cur[:, ks, 1],
                                                o[:, qs], lse[:, :, qs].contiguous(), rel, scale)
                    dq[:, qs] += dq_p
                    acc[:, ks, 0] += dk_p
                    acc[:, ks, 1] += dv_p
            # the accumulator follows its block (after the last step it is home)
            if cp > 1:
                acc_in = torch.empty_like(acc)
                for rq in _exchange([acc], [acc_in], group):
                    rq.wait()
                acc = acc_in
            if reqs is not None:
                for rq in reqs:
                    rq.wait()
                cur = nxt
        dk = acc[:, :, 0].to(q.dtype)
        dv = acc[:, :, 1].to(q.dtype)
        return dq.to(q.dtype), dk, dv, None, None, None


def ring_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, group,
                   scale: Optional[float] = None) -> torch.Tensor:
    """q [B, 2c, Hq, D], k/v [B, 2c, Hk, D]: this rank's zigzag tokens (after
    QK-norm and RoPE at their global positions) -> attention output
    [B, 2c, Hq, D], causal over the whole sequence."""
    D = q.shape[-1]
    scale = scale if scale is not None else 1.0 / math.sqrt(D)
    if q.shape[1] % 2:
        raise ValueError("ring attention needs the zigzag layout (two equal chunks per rank)")
    pair = KernelPair() if q.is_cuda else TorchPair()
    return _RingFn.apply(q, k, v, group, float(scale), pair)


class _QKNormRope(torch.autograd.Function):
    """QK-RMSNorm + RoPE on the sm_100a kernels with their backward:
    qkv [B, S, (Hq+2Hk)*D] -> q [B,S,Hq,D], k [B,S,Hk,D], v [B,S,Hk,D]."""

    @staticmethod
    def forward(ctx, qkv, q_w, k_w, cos, sin, pos, Hq, Hk, D, eps):
        from ..ops._ext import ext
        B, S, _ = qkv.shape
        qkv2 = qkv.reshape(B * S, -1).contiguous()
        pos1 = pos.reshape(-1).contiguous()
        qk, rstd = ext().qknorm_rope_fwd(qkv2, q_w, k_w, cos, sin, pos1, B, S, Hq, Hk, D, float(eps))
        ctx.save_for_backward(qkv2, rstd, q_w, k_w, cos, sin, pos1)
        ctx.meta = (B, S, Hq, Hk, D)
        q = qk[:, :Hq * D].reshape(B, S, Hq, D)
        k = qk[:, Hq * D:].reshape(B, S, Hk, D)
        v = qkv2[:, (Hq + Hk) * D:].reshape(B, S, Hk, D)
        return q, k, v

    @staticmethod
    def backward(ctx, dq, dk, dv):
        from ..ops._ext import ext
        from ..ops.common import grad_buffer
        qkv2, rstd, q_w, k_w, cos, sin, pos = ctx.saved_tensors
        B, S, Hq, Hk, D = ctx.meta
        T = B * S
        dqk = torch.cat([dq.reshape(T, Hq * D).float(), dk.reshape(T, Hk * D).float()], 1).contiguous()
        dqkv = torch.empty_like(qkv2)
        dqkv[:, (Hq + Hk) * D:] = dv.reshape(T, Hk * D).to(dqkv.dtype)
        dqw = grad_buffer(q_w) if (q_w is not None and q_w.requires_grad) else None
        dkw = grad_buffer(k_w) if (k_w is not None and k_w.requires_grad) else None
        ext().qknorm_rope_bwd(dqk, qkv2, q_w, k_w, rstd, cos, sin, pos, dqkv, dqw, dkw,
                              B, S, Hq, Hk, D)
        return (dqkv.view(B, S, -1),) + (None,) * 9


def ring_attention_qkv(qkv, q_w, k_w, cos, sin, pos, group, Hq, Hk, D, eps,
                       scale: Optional[float] = None) -> torch.Tensor:
    """Projected qkv [B, 2c, (Hq+2Hk)*D] of this rank's zigzag tokens at global
    positions ``pos`` [B, 2c] -> attention output [B, 2c, Hq*D]."""
    B, S, _ = qkv.shape
    if qkv.is_cuda:
        q, k, v = _QKNormRope.apply(qkv, q_w, k_w, cos, sin, pos.to(torch.int64), Hq, Hk, D, eps)
    else:
        from ..ops import reference as ref
        q, k, v = qkv.split([Hq * D, Hk * D, Hk * D], dim=-1)
        q = q.reshape(B, S, Hq, D)
        k = k.reshape(B, S, Hk, D)
        v = v.reshape(B, S, Hk, D)
        q, k = ref.qk_norm_rope(q, k, q_w, k_w, cos[pos], sin[pos], eps)
    return ring_attention(q, k, v, group, scale).reshape(B, S, Hq * D)
