"""Data parallelism over the flat parameter store.

Two modes, both operating on slices of the ``FlatParamStore`` buffers (no
packing copies):

* ``replicate``: every rank keeps full weights/optimizer state; gradients are
  averaged with bucketed all-reduces after the backward pass.
* ``shard`` (default; the role FSDP2 plays in the reference,
  reference: distributed/fsdp.py:44-75): gradients are reduce-scattered so each
  rank owns 1/N of the flat buffer, the fused AdamW kernel updates only that
  shard, and the updated bf16 compute copy is all-gathered.  This is ZeRO-2:
  with 180 GB of HBM per B200 the bf16 working copy of every model in the
  benchmark configurations fits, so the forward needs no per-layer parameter
  all-gather at all; the fp32 master/Adam state (16 B/param) is what gets
  sharded.

Under expert parallelism the store's expert span holds different experts on
the ranks of different EP blocks: shard mode then splits the store into
three pieces with equal shards each (the store pads the span's ends for
that): the dense pieces before and after the span over this group, the span
over the ranks that hold the same experts, and the optimizer keeps its
moments for the owned ranges only.

Shard boundaries are multiples of 64 elements.  The Adam moments exist only
for the shard (see ``FusedAdamW``); ``gather_master`` / ``gather_flat_``
all-gather the fp32 master weights and the moments before a full state-dict
save.
"""

from __future__ import annotations

from typing import Tuple

import torch
import torch.distributed as dist

from ..runtime.flat_params import ALIGN, FlatParamStore
from .comm import (all_gather_flat_, all_reduce_avg_, get_rank, get_world_size,
                   reduce_scatter_avg_)


def shard_bounds(numel: int, world: int, rank: int) -> Tuple[int, int]:
    per = (numel + world - 1) // world
    per = (per + ALIGN - 1) // ALIGN * ALIGN
    b = min(numel, rank * per)
    e = min(numel, b + per)
    return b, e


def _src(group) -> int:
    """Global rank of the group's first member (``dist.broadcast`` takes a
    global rank)."""
    return dist.get_global_rank(group, 0) if group is not None else 0


class DataParallel:
    """``expert_group``: ranks that hold the same experts under expert
    parallelism (one per EP block).  The store's expert span is summed over it
    and divided by the data-parallel world, which equals the data-parallel mean
    of the full-batch expert gradient (each EP rank's expert gradient already
    sums the tokens of its whole EP block).  In shard mode the span is also
    sharded over that group (three pieces, ``split``)."""

    def __init__(self, store: FlatParamStore, mode: str = "shard", group=None,
                 bucket_mb: float = 256.0, expert_group=None):
        self.store = store
        self.group = group
        xb, xe = getattr(store, "expert_span", (0, 0))
        self.expert_span = (xb, xe) if xe > xb else None
        self.expert_group = expert_group
        self.mode = mode
        self.world = get_world_size(group)
        self.rank = get_rank(group)
        self.per = shard_bounds(store.numel, self.world, 0)[1]
        self.padded = self.per * self.world
        self.shard = shard_bounds(store.numel, self.world, self.rank) if mode == "shard" else (0, store.numel)
        # shard mode with an expert span: the dense pieces before and after
        # the span are sharded over this group, the span over the ranks
        # holding the same experts (each owner's expert gradient already sums
        # its EP block's tokens: sum over those ranks, divide by this world)
        self.split = None
        if self.expert_span is not None and mode == "shard" and self.world > 1:
            xg = expert_group if expert_group is not None and get_world_size(expert_group) > 1 else None
            xw = get_world_size(xg) if xg is not None else 1
            xr = get_rank(xg) if xg is not None else 0
            self.split = [(0, xb, group, self.world, self.rank, 1.0),
                          (xe, store.numel, group, self.world, self.rank, 1.0),
                          (xb, xe, xg, xw, xr, xw / self.world)]
        # the optimizer keeps its state for ``owned_ranges()`` back to back
        self.piecewise = self.split is not None
        self.bucket_elems = max(ALIGN, int(bucket_mb * 1024 * 1024 / 4) // ALIGN * ALIGN)
        # Reduce-scatter / all-gather need equal chunks: pad the flat buffers' views.
        self._grad_pad = None
        self._comp_pad = None
        self._master_pad = None

    # -------------------------------------------------------------- helpers
    def _padded(self, buf: torch.Tensor, cache_attr: str) -> torch.Tensor:
        if buf.numel() >= self.padded:
            return buf[: self.padded]
        cached = getattr(self, cache_attr)
        if cached is None or cached.numel() != self.padded or cached.dtype != buf.dtype:
            cached = torch.zeros(self.padded, dtype=buf.dtype, device=buf.device)
            setattr(self, cache_attr, cached)
        cached[: buf.numel()].copy_(buf)
        return cached

    # ---------------------------------------------------------------- pieces
    @staticmethod
    def _owned(lo, hi, w, r):
        per = shard_bounds(hi - lo, w, 0)[1]
        return lo + min(hi - lo, r * per), lo + min(hi - lo, (r + 1) * per), per

    def owned_ranges(self):
        """The flat ranges this rank reduces and updates."""
        if self.split is None:
            return [self.shard]
        out = []
        for lo, hi, _, w, r, _ in self.split:
            b, e, _ = self._owned(lo, hi, w, r)
            if e > b:
                out.append((b, e))
        return out

    def _piece_rs(self, g, lo, hi, grp, w, r, scale) -> None:
        """Mean over ``grp`` of g[lo:hi], this rank's share written in place."""
        b, e, per = self._owned(lo, hi, w, r)
        if w > 1 and hi > lo:
            src = g[lo:hi]
            if per * w != hi - lo:
                src = torch.zeros(per * w, dtype=g.dtype, device=g.device)
                src[:hi - lo].copy_(g[lo:hi])
            out = src[r * per:(r + 1) * per]
            reduce_scatter_avg_(out, src, grp)
            if src.data_ptr() != g[lo:hi].data_ptr():
                g[b:e].copy_(out[:e - b])
        if scale != 1.0 and e > b:
            g[b:e].mul_(scale)

    def _piece_ag(self, buf, lo, hi, grp, w, r) -> None:
        """Complete buf[lo:hi] over ``grp`` from each rank's share."""
        if w == 1 or hi <= lo:
            return
        b, e, per = self._owned(lo, hi, w, r)
        if per * w == hi - lo:
            bp = buf[lo:hi]
            all_gather_flat_(bp, bp[r * per:(r + 1) * per].clone(), grp)
            return
        bp = torch.zeros(per * w, dtype=buf.dtype, device=buf.device)
        bp[r * per:r * per + (e - b)].copy_(buf[b:e])
        all_gather_flat_(bp, bp[r * per:(r + 1) * per].clone(), grp)
        buf[lo:hi].copy_(bp[:hi - lo])

    # --------------------------------------------------------------- overlap
    def attach_overlap(self, model) -> None:
        """Shard mode without an expert span: reduce-scatter each transformer
        block's (decay) gradient span as soon as the block's backward is done
        on the last micro-batch, on a side stream next to the rest of the
        backward; the remaining ranges after the backward.  Ownership becomes
        per span (each span split into equal shards), so this is attached
        before the optimizer is built (``piecewise``)."""
        if self.mode != "shard" or self.world == 1 or self.split is not None:
            return
        from ..models.transformer import TransformerBlock
        st = self.store
        spans = []
        for blk in model.modules():
            if not isinstance(blk, TransformerBlock):
                continue
            ps = [p for p in blk.parameters() if id(p) in st.offsets
                  and st.offsets[id(p)] < st.decay_end]
            if not ps:
                continue
            lo = min(st.offsets[id(p)] for p in ps) // ALIGN * ALIGN
            hi = (max(st.offsets[id(p)] + p.numel() for p in ps) + ALIGN - 1) // ALIGN * ALIGN
            mine = {id(p) for p in ps}
            if any(id(q) not in mine and lo <= st.offsets[id(q)] < hi for q in st.params):
                continue  # not contiguous: reduced with the rest
            spans.append((lo, hi, blk))
        spans.sort(key=lambda t: t[0])
        pieces, hooks, pos = [], {}, 0
        for lo, hi, blk in spans:
            if lo < pos:
                continue
            if lo > pos:
                pieces.append((pos, lo))
            hooks[len(pieces)] = blk
            pieces.append((lo, hi))
            pos = hi
        if pos < st.numel:
            pieces.append((pos, st.numel))
        self.split = [(lo, hi, self.group, self.world, self.rank, 1.0) for lo, hi in pieces]
        self.piecewise = True
        self._hooked = set(hooks)
        self._issued, self._final = set(), False
        self._stream = torch.cuda.Stream(device=st.grad.device) if st.grad.is_cuda else None
        for k, blk in hooks.items():
            blk.grad_ready_hook = self._make_hook(k)

    def _make_hook(self, k: int):
        def hook():
            if not self._final or k in self._issued:
                return
            self._issued.add(k)
            lo, hi, grp, w, r, scale = self.split[k]
            if self._stream is None:
                self._piece_rs(self.store.grad, lo, hi, grp, w, r, scale)
                return
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream())
            self._stream.wait_event(ev)
            with torch.cuda.stream(self._stream):
                self._piece_rs(self.store.grad, lo, hi, grp, w, r, scale)
        return hook

    def begin_step(self, final_micro: bool) -> None:
        """Called by the engine before each micro-batch's backward: the
        block hooks reduce only on the last one."""
        if getattr(self, "_hooked", None) is None:
            return
        if final_micro and not self._final:
            self._issued = set()
        self._final = final_micro

    # ------------------------------------------------------------- gradients
    @torch.no_grad()
    def sync_grads(self) -> None:
        if self.world == 1:
            return
        g = self.store.grad
        if self.split is not None:
            hooked = getattr(self, "_hooked", None)
            if hooked is not None and self._stream is not None:
                torch.cuda.current_stream().wait_stream(self._stream)
            issued = self._issued if (hooked is not None and self._final) else set()
            self.last_overlapped = len(issued)   # spans reduced during the backward
            for k, (lo, hi, grp, w, r, scale) in enumerate(self.split):
                if k not in issued:
                    self._piece_rs(g, lo, hi, grp, w, r, scale)
            if hooked is not None:
                self._issued, self._final = set(), False
            return
        if self.mode == "replicate":
            for b, e in self._dense_ranges(g.numel()):
                for s in range(b, e, self.bucket_elems):
                    all_reduce_avg_(g[s:min(e, s + self.bucket_elems)], self.group)
            if self.expert_span is not None:
                xb, xe = self.expert_span
                if self.expert_group is not None and get_world_size(self.expert_group) > 1:
                    dist.all_reduce(g[xb:xe], group=self.expert_group)
                g[xb:xe].mul_(1.0 / self.world)
            return
        gp = self._padded(g, "_grad_pad")
        out = gp[self.rank * self.per:(self.rank + 1) * self.per]
        reduce_scatter_avg_(out, gp, self.group)
        if gp.data_ptr() != g.data_ptr():
            b, e = self.shard
            g[b:e].copy_(gp[b:e])

    def _dense_ranges(self, n: int):
        if self.expert_span is None:
            return [(0, n)]
        xb, xe = self.expert_span
        return [(0, xb), (xe, n)]

    def norm_sq_reduce(self, sq: torch.Tensor) -> torch.Tensor:
        """Global squared gradient norm from this rank's part.

        Shard mode: each rank holds a disjoint shard, so the parts add up.
        Replicate mode with an expert span (expert parallelism): the dense
        gradient is the same on every rank after the reduction, but each rank
        holds other experts, so the expert part is summed over the group and
        divided by the number of ranks holding each expert set.  Without that,
        every rank would clip with its own norm and the replicated weights
        would drift apart."""
        if self.world <= 1:
            return sq
        if self.mode == "shard":
            sq = sq.clone()
            dist.all_reduce(sq, group=self.group)
        elif self.expert_span is not None:
            xb, xe = self.expert_span
            g = self.store.grad[xb:xe]
            if g.is_cuda:
                from ..ops._ext import ext
                part = ext().sum_squares(g).reshape(sq.shape)
            else:
                part = torch.linalg.vector_norm(g).square().reshape(sq.shape)
            tot = part.clone()
            dist.all_reduce(tot, group=self.group)
            reps = get_world_size(self.expert_group) if self.expert_group is not None else 1
            sq = sq - part + tot / reps
        return sq

    # ------------------------------------------------------------ parameters
    @torch.no_grad()
    def gather_params(self) -> None:
        """All-gather the updated compute copy after a sharded optimizer step."""
        if self.world == 1 or self.mode != "shard":
            return
        st = self.store
        buf = st.compute if st.compute is not None else st.master
        if self.split is not None:
            for lo, hi, grp, w, r, _ in self.split:
                self._piece_ag(buf, lo, hi, grp, w, r)
            if st.compute is not None:
                self.sync_fp32_span()
            return
        bp = self._padded(buf, "_comp_pad")
        mine = bp[self.rank * self.per:(self.rank + 1) * self.per]
        if bp.data_ptr() != buf.data_ptr():
            b, e = self.shard
            mine[: e - b].copy_(buf[b:e])
        all_gather_flat_(bp, mine.clone(), self.group)
        if bp.data_ptr() != buf.data_ptr():
            buf.copy_(bp[: buf.numel()])
        if st.compute is not None:
            self.sync_fp32_span()

    @torch.no_grad()
    def sync_fp32_span(self) -> None:
        """Make the master's fp32-read span (norm weights, biases) complete on
        every rank after a sharded update: each rank contributes its shard's
        part, summed with one small all-reduce."""
        lo, hi = getattr(self.store, "fp32_span", (0, 0))
        if self.world == 1 or self.mode != "shard" or hi <= lo:
            return
        m = self.store.master
        buf = getattr(self, "_span_buf", None)
        if buf is None or buf.numel() != hi - lo:
            buf = self._span_buf = torch.zeros(hi - lo, dtype=torch.float32, device=m.device)
        buf.zero_()
        for b, e in self.owned_ranges():
            ib, ie = max(lo, b), min(hi, e)
            if ie > ib:
                buf[ib - lo:ie - lo].copy_(m[ib:ie])
        dist.all_reduce(buf, group=self.group)
        m[lo:hi].copy_(buf)

    @torch.no_grad()
    def gather_master(self) -> None:
        self.gather_flat_(self.store.master)

    @torch.no_grad()
    def gather_flat_(self, buf: torch.Tensor) -> None:
        """All-gather a store-sized fp32 buffer in which each rank holds its
        own shard [b, e) (in place): the master weights, or the Adam moments
        before a checkpoint save."""
        if self.world == 1 or self.mode != "shard":
            return
        if self.split is not None:
            for lo, hi, grp, w, r, _ in self.split:
                self._piece_ag(buf, lo, hi, grp, w, r)
            return
        bp = self._padded(buf, "_master_pad")
        mine = bp[self.rank * self.per:(self.rank + 1) * self.per].clone()
        all_gather_flat_(bp, mine, self.group)
        if bp.data_ptr() != buf.data_ptr():
            buf.copy_(bp[: buf.numel()])

    @torch.no_grad()
    def broadcast_params(self, src: int = 0) -> None:
        """Make every rank start from rank ``src``'s weights."""
        if self.world == 1:
            return
        m = self.store.master
        if self.expert_span is None:
            dist.broadcast(m, src=_src(self.group), group=self.group)
        else:
            for b, e in self._dense_ranges(m.numel()):
                t = m[b:e].clone()
                dist.broadcast(t, src=_src(self.group), group=self.group)
                m[b:e].copy_(t)
            if self.expert_group is not None and get_world_size(self.expert_group) > 1:
                xb, xe = self.expert_span
                t = m[xb:xe].clone()
                dist.broadcast(t, src=_src(self.expert_group), group=self.expert_group)
                m[xb:xe].copy_(t)
        self.store.refresh_compute()
