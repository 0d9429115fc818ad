"""Data parallelism whose optimizer step moves its bulk traffic with this
library's own kernels over NVLink peer memory (``csrc/zero_comm.cu``).

The flat store's gradient buffer (fp32) and compute copy (bf16) are allocated
in symmetric memory (``torch.distributed._symmetric_memory``: every rank's
buffer is mapped into every peer's address space; only the pointer exchange
comes from PyTorch).  One step is:

1. ``zero_rs``: signal/wait on peer flags, then each rank reads its shard of
   every peer's gradient with P2P loads, writes the mean and accumulates the
   squared norm (reduce-scatter fused with the 1/world scale and the norm);
2. a 4-byte all-reduce of the squared norm (NCCL) and the clip factor;
3. ``zero_adamw_ag``: sharded AdamW whose bf16 result is stored straight into
   every peer's compute copy (all-gather fused into the optimizer);
4. ``zero_publish``: flag barrier so the next forward reads complete weights.

The Adam moments are allocated for this rank's shard only; the fp32 master
is updated only in the shard (the rest is refreshed by ``gather_master``
before a save).  Same interface as ``DataParallel``; the engine calls
``fused_step`` instead of sync + clip + step + gather.  Requires 1, 2, 4 or 8
ranks on one NVSwitch domain.

Under expert parallelism the store's expert span holds different experts on
the ranks of different expert blocks, so it is reduced and updated only over
the ranks that hold the same experts (``expert_group``, a subset of the
data-parallel group): its own shard bounds, its own flag words and the
subset of the peer pointers the data-parallel mapping already provides.  The
dense shard skips the expert span (always as two reduce calls, possibly
empty, so every rank issues the same sequence of flag epochs).
"""

from __future__ import annotations

import importlib
import os
from typing import List

import torch
import torch.distributed as dist

from ..ops._ext import ext
from ..runtime.flat_params import ALIGN, FlatParamStore
from .comm import all_gather_flat_, get_world_size
from .data_parallel import DataParallel, shard_bounds


def same_node(ranks: List[int], local_world_size: int) -> bool:
    """True when every global rank in ``ranks`` runs on one node, with
    ``local_world_size`` consecutive ranks per node (torchrun's layout); an
    unknown size (0) means a single-node launch."""
    if local_world_size <= 0:
        return True
    return len({r // local_world_size for r in ranks}) == 1


def symmetric_available(group=None) -> bool:
    """Peer-memory kernels need NCCL ranks of one NVLink domain: 2, 4 or 8
    ranks on the same node (a group that spans nodes falls back to NCCL)."""
    if not (torch.cuda.is_available() and dist.is_initialized()):
        return False
    if dist.get_backend(group) != "nccl" or get_world_size(group) not in (2, 4, 8):
        return False
    ranks = (dist.get_process_group_ranks(group) if group is not None
             else list(range(dist.get_world_size())))
    if not same_node(ranks, int(os.environ.get("LOCAL_WORLD_SIZE", "0") or 0)):
        return False
    try:
        importlib.import_module("torch.distributed._symmetric_memory")
        return True
    except Exception:
        return False


class SymmetricAllocator:
    """``alloc(numel, dtype, device)`` for ``FlatParamStore``: zero-filled
    tensors in symmetric memory."""

    def __init__(self, group=None):
        symm = importlib.import_module("torch.distributed._symmetric_memory")
        self.symm = symm
        self.group = group or dist.group.WORLD
        self.group_name = self.group.group_name
        enable = getattr(symm, "enable_symm_mem_for_group", None)
        if enable is not None:
            try:
                enable(self.group_name)
            except Exception:
                pass
        self.tensors: List[torch.Tensor] = []

    def __call__(self, numel: int, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
        t = self.symm.empty(numel, dtype=dtype, device=device)
        t.zero_()
        self.tensors.append(t)
        return t

    def peer_ptrs(self, t: torch.Tensor) -> List[int]:
        h = self.symm.rendezvous(t, self.group_name)
        self.handles = getattr(self, "handles", []) + [h]  # keep the mappings alive
        return [int(p) for p in h.buffer_ptrs]


def _group_ranks(group) -> List[int]:
    return (dist.get_process_group_ranks(group) if group is not None
            else list(range(dist.get_world_size())))


class PeerDataParallel(DataParallel):
    def __init__(self, store: FlatParamStore, allocator: SymmetricAllocator, group=None,
                 rs_ctas: int = 0, expert_group=None):
        super().__init__(store, mode="shard", group=group, expert_group=expert_group)
        self.mode = "shard"
        self.shard = shard_bounds(store.numel, self.world, self.rank)
        # its own layout: the dense shard over the whole store, skipping the
        # expert span, and the span's shard over the expert ranks
        self.split = None
        self.piecewise = True
        self.alloc = allocator
        dev = store.master.device
        self.flags = allocator(2 * 8, torch.int32, dev)
        self.xflags = allocator(2 * 8, torch.int32, dev) if self.expert_span is not None else None
        torch.cuda.synchronize()
        self.p_grad = allocator.peer_ptrs(store.grad)
        self.p_comp = allocator.peer_ptrs(store.compute)
        self.p_flags = allocator.peer_ptrs(self.flags)
        self.x_shard = None
        if self.xflags is not None:
            p_xflags = allocator.peer_ptrs(self.xflags)
            dp_ranks = _group_ranks(group)
            me = dist.get_rank()
            members = _group_ranks(expert_group) if expert_group is not None else [me]
            idx = [dp_ranks.index(r) for r in members]
            self.x_rank, self.x_world = members.index(me), len(members)
            self.x_grad = [self.p_grad[i] for i in idx]
            self.x_comp = [self.p_comp[i] for i in idx]
            self.x_flags = [p_xflags[i] for i in idx]
            xb, xe = self.expert_span
            lo, hi = shard_bounds(xe - xb, self.x_world, self.x_rank)
            self.x_shard = (xb + lo, xb + hi)
            self.x_per = shard_bounds(xe - xb, self.x_world, 0)[1]
            fb, fe = getattr(store, "fp32_span", (0, 0))
            if fe > fb and fb < xe and xb < fe:
                raise ValueError("the fp32 span overlaps the expert span")
        dist.barrier(group=group)
        self.epoch = 0
        self.x_epoch = 0
        self.rs_ctas = rs_ctas
        self.sq = torch.zeros(1, dtype=torch.float32, device=dev)
        self.norm = torch.zeros((), dtype=torch.float32, device=dev)
        self.clip = torch.ones((), dtype=torch.float32, device=dev)

    # ------------------------------------------------------------ overlap
    def attach_overlap(self, model, ctas: int = 16) -> None:
        """Reduce each transformer block's gradient span on a side stream as
        soon as the block's backward is done (last micro-batch only), with a
        small grid that shares the SMs with the backward kernels."""
        from ..models.transformer import TransformerBlock
        if self.expert_span is not None:
            return  # expert spans are reduced after the backward
        st = self.store
        spans = []
        for blk in model.modules():
            if not isinstance(blk, TransformerBlock):
                continue
            ps = [p for p in blk.parameters() if id(p) in st.offsets
                  and st.offsets[id(p)] < st.decay_end]
            if not ps:
                continue
            lo = min(st.offsets[id(p)] for p in ps)
            hi = max(st.offsets[id(p)] + p.numel() for p in ps)
            mine = {id(p) for p in ps}
            others = [q for q in st.params if id(q) not in mine and lo <= st.offsets[id(q)] < hi]
            if others:
                continue  # not contiguous: reduced with the remainder at the end
            lo = lo // ALIGN * ALIGN
            hi = (hi + ALIGN - 1) // ALIGN * ALIGN
            spans.append((lo, hi))
            blk.grad_ready_hook = self._make_hook(len(spans) - 1)
        self.spans = spans
        self.overlap_ctas = ctas
        self.comm_stream = torch.cuda.Stream(device=st.master.device)
        self.final_micro = False
        cover = sorted(spans)
        rest, pos = [], 0
        for lo, hi in cover:
            if lo > pos:
                rest.append((pos, lo))
            pos = max(pos, hi)
        if pos < st.numel:
            rest.append((pos, st.numel))
        self.rest = rest

    def _make_hook(self, k: int):
        def hook():
            if not self.final_micro or k in self._issued:
                return
            self._issued.add(k)
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream())
            self.comm_stream.wait_event(ev)
            with torch.cuda.stream(self.comm_stream):
                self._rs(*self.spans[k], self.overlap_ctas)
        return hook

    def begin_step(self, final_micro: bool) -> None:
        """Called by the engine before each micro-batch's backward."""
        if getattr(self, "spans", None) is None:
            return
        if final_micro and not self.final_micro:
            self._issued = set()
            self.sq.zero_()
            self._calls = 0
        self.final_micro = final_micro

    def _rs(self, lo: int, hi: int, ctas: int) -> None:
        b, e = self.shard
        lo, hi = max(lo, b), min(hi, e)
        if hi < lo:
            hi = lo
        self._calls += 1
        ext().zero_rs(self.p_grad, self.p_comp, self.p_flags, self.rank, lo, hi, self.sq,
                      self.epoch + self._calls, ctas, 1.0)

    def dense_pieces(self, lo: int, hi: int):
        """[lo, hi) without the expert span: two ranges, either possibly empty."""
        if self.expert_span is None:
            return [(lo, hi)]
        xb, xe = self.expert_span
        return [(lo, min(hi, xb)), (max(lo, xe), hi)]

    def owned_ranges(self):
        """The flat ranges this rank reduces and updates."""
        b, e = self.shard
        out = [(lo, hi) for lo, hi in self.dense_pieces(b, e) if hi > lo]
        if self.x_shard is not None and self.x_shard[1] > self.x_shard[0]:
            out.append(self.x_shard)
        return out

    def sync_grads(self) -> None:
        """Reduce-scatter whatever the overlapped block reductions did not
        cover (everything, without ``attach_overlap``)."""
        if getattr(self, "spans", None) is None:
            self._calls = 0
            self.sq.zero_()
            for lo, hi in self.dense_pieces(0, self.store.numel):
                self._rs(lo, hi, self.rs_ctas)
            if self.x_shard is not None:
                self.x_epoch += 1
                xb, xe = self.x_shard
                # each expert's gradient already sums the tokens its EP block
                # routed to it: sum over the ranks holding the same experts and
                # divide by the data-parallel world (x_world / world x mean)
                ext().zero_rs(self.x_grad, self.x_comp, self.x_flags, self.x_rank, xb, xe,
                              self.sq, self.x_epoch, self.rs_ctas, self.x_world / self.world)
        else:
            torch.cuda.current_stream().wait_stream(self.comm_stream)
            if not self.final_micro:  # no backward ran with the hooks armed
                self._issued, self._calls = set(), 0
                self.sq.zero_()
            missing = [self.spans[k] for k in range(len(self.spans)) if k not in self._issued]
            for lo, hi in missing + self.rest:
                self._rs(lo, hi, self.rs_ctas)
            self.final_micro = False
        self.epoch += self._calls

    @torch.no_grad()
    def fused_step(self, optimizer, max_norm: float, extra_sq=None) -> torch.Tensor:
        """Reduce-scatter + norm, clip, sharded AdamW + all-gather, publish.
        Returns the global gradient norm (device tensor)."""
        E = ext()
        self.sync_grads()
        sq = self.sq
        if extra_sq is not None:
            sq = extra_sq(sq)
        dist.all_reduce(sq, group=self.group)
        E.zero_clip(sq, float(max_norm or 0.0), self.clip, self.norm)
        optimizer.clip_scale = self.clip
        optimizer.last_grad_norm = self.norm

        def update(hp):
            lr_d, lr_n, b1, b2, eps, wd, bc1, bc2 = hp
            # the optimizer's state is this rank's owned ranges back to back
            for lo, hi, off in optimizer.pieces:
                expert = self.x_shard is not None and (lo, hi) == self.x_shard
                ptrs = ((self.x_grad, self.x_comp, self.x_flags, self.x_rank) if expert
                        else (self.p_grad, self.p_comp, self.p_flags, self.rank))
                E.zero_adamw_ag(*ptrs, self.store.master, optimizer.exp_avg[off:],
                                optimizer.exp_avg_sq[off:], self.clip, lo, hi, lo,
                                self.store.decay_end, lr_d, lr_n, b1, b2, eps, wd, bc1, bc2)

        optimizer.step(update=update)
        E.zero_publish(self.p_grad, self.p_comp, self.p_flags, self.rank, self.epoch)
        self.sync_fp32_span()
        return self.norm

    def gather_params(self) -> None:
        """The fused step already wrote every peer's compute copy."""
        return

    @torch.no_grad()
    def gather_flat_(self, buf: torch.Tensor) -> None:
        """Complete a store-sized fp32 buffer of which this rank holds its
        owned ranges: the dense shards over the data-parallel group, then the
        expert span over the ranks holding the same experts."""
        if self.x_shard is None:
            return super().gather_flat_(buf)
        xb, xe = self.x_shard
        mine = buf[xb:xe].clone()
        super().gather_flat_(buf)
        sb = self.expert_span[0]
        full = torch.zeros(self.x_per * self.x_world, dtype=buf.dtype, device=buf.device)
        if self.x_world > 1:
            part = torch.zeros(self.x_per, dtype=buf.dtype, device=buf.device)
            part[:xe - xb].copy_(mine)
            all_gather_flat_(full, part, self.expert_group)
        else:
            full[:xe - xb].copy_(mine)
        n = self.expert_span[1] - sb
        buf[sb:sb + n].copy_(full[:n])
