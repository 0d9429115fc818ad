"""Fully sharded data parallelism: weights, gradients and optimizer state are
all sharded over the data-parallel group, and each transformer block's
weights exist in full only while that block runs (the role of FSDP2's
``fully_shard`` per block with ``reshard_after_forward=True``, bf16 gathers
and fp32 gradient reduction; reference: distributed/fsdp.py:36-75).

Layout.  The trainable parameters are grouped into *units*:

* one per transformer block (its matrices; freed after the block's forward
  and backward),
* one for the other decayed matrices (lm_head when untied),
* one for the non-decayed matrices (the embedding table),
* one for every 1-D parameter (norm weights, biases), kept in fp32 because
  the norm kernels read fp32 weights.

The last three stay gathered for a whole training step.  A unit is a flat
buffer padded to a multiple of 64 x world elements (fusion groups such as
q|k|v and gate|up contiguous, 64-element aligned, as in ``FlatParamStore``);
rank r owns the r-th contiguous 1/world of every unit.  Per rank the store
keeps only its shards: ``master`` and ``grad`` (fp32), ``compute`` (the
compute dtype, bf16 on the GPU: what the all-gathers read; the fused AdamW
kernel writes it) and, in ``FSDPAdamW``, the two Adam moments, so weights,
gradients and optimizer state cost 18 B per parameter / world.

Schedule of a block unit:

* forward: all-gather the unit (the next block's gather is issued at the same
  time, asynchronously), run the block, release the gathered buffer;
* backward: all-gather again (prefetching the previous block), allocate a
  zeroed fp32 gradient buffer that the weight-gradient GEMMs accumulate into,
  and when the gradient reaches the block's input reduce-scatter it (mean
  over ranks) on a side stream into the gradient shard and release both
  buffers.

The persistent units accumulate their gradients over the micro-batches of a
step and are reduce-scattered once after the last one.  Parameters are views
of the gathered buffers (their storage is resized to zero while a unit is
released, so the views made at construction stay valid); module code,
``state_dict`` and the GEMMs' weight views keep working across gathers.
``FSDPAdamW.gather_full_state`` rebinds the parameters to full fp32 tensors
for checkpointing, so a checkpoint holds the single-process model's names and
shapes and loads into any other layout.

Collectives are torch.distributed's (NCCL on GPUs, Gloo in the CPU tests):
this is the sharding and scheduling layer; the peer-memory ZeRO step
(``parallel.peer_dp``) remains the faster choice when the bf16 weights fit on
every GPU.
"""

from __future__ import annotations

import contextlib
from typing import Dict, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist
import torch.nn as nn

from ..runtime.flat_params import ALIGN, default_groups, no_decay_rule
from ..training.optimizer import FusedAdamW
from .comm import all_gather_flat_, get_rank, get_world_size, is_dist, reduce_scatter_avg_

_FREE, _GATHERING, _READY = 0, 1, 2


def _set_storage(t: torch.Tensor, numel: int) -> None:
    """Allocate (numel > 0) or release (0) the storage behind ``t``; views
    made while it was allocated stay valid."""
    st = t.untyped_storage()
    nbytes = numel * t.element_size()
    if st.nbytes() != nbytes:
        st.resize_(nbytes)


def partition(model: nn.Module):
    """Group the trainable parameters into units: (blocks, per-block dense
    fusion groups, per-block expert fusion groups, other decayed matrices,
    non-decayed matrices, 1-D parameters)."""
    from ..models.transformer import TransformerBlock
    groups = [g for g in default_groups(model) if all(p.requires_grad for _, p in g)]
    blocks = [m for m in model.modules() if isinstance(m, TransformerBlock)]
    owner: Dict[int, int] = {}
    for bi, blk in enumerate(blocks):
        for p in blk.parameters():
            owner.setdefault(id(p), bi)
    per_block: List[list] = [[] for _ in blocks]
    per_block_experts: List[list] = [[] for _ in blocks]
    rest_decay, rest_nodecay, small = [], [], []
    for grp in groups:
        # a fusion group is homogeneous in rank and decay; split it if not
        kinds = {(p.ndim <= 1, no_decay_rule(n, p), bool(getattr(p, "_ep_local", False)))
                 for n, p in grp}
        parts = [grp] if len(kinds) == 1 else [[item] for item in grp]
        for part in parts:
            n0, p0 = part[0]
            expert = bool(getattr(p0, "_ep_local", False))
            if expert and (p0.ndim <= 1 or no_decay_rule(n0, p0) or id(p0) not in owner):
                raise NotImplementedError(f"expert-parallel parameter {n0} outside the "
                                          "blocks' expert matrices")
            if p0.ndim <= 1:
                small.append(part)
            elif no_decay_rule(n0, p0):
                rest_nodecay.append(part)
            elif expert:
                per_block_experts[owner[id(p0)]].append(part)
            elif id(p0) in owner:
                per_block[owner[id(p0)]].append(part)
            else:
                rest_decay.append(part)
    return blocks, per_block, per_block_experts, rest_decay, rest_nodecay, small


class ParamUnit:
    """One flat buffer of parameters gathered and released together, sharded
    over its own process group (the data-parallel group; for expert-parallel
    experts the group of ranks that hold the same experts)."""

    def __init__(self, name: str, groups, dtype: torch.dtype, persistent: bool, decay: bool,
                 group=None, grad_scale: float = 1.0, local: bool = False,
                 world: Optional[int] = None):
        """``local``: not sharded (this rank alone holds these parameters).
        ``world``: shard count to plan with, without a process group."""
        self.name = name
        self.dtype = dtype
        self.persistent = persistent
        self.decay = decay
        self.group = group
        self.world = 1 if local else (world if world is not None else get_world_size(group))
        self.rank = 0 if local else (0 if world is not None else get_rank(group))
        self.distributed = is_dist() and self.world > 1
        self.nccl = self.distributed and dist.get_backend(group) == "nccl"
        # multiplies the mean over ``group`` of the gradient (experts: the
        # data-parallel mean is the sum over the group / data-parallel world)
        self.grad_scale = grad_scale
        self.params: List[nn.Parameter] = []
        self.names: List[str] = []
        self.local: Dict[int, int] = {}
        self.groups: List[List[nn.Parameter]] = []
        off = 0
        for grp in groups:
            off = (off + ALIGN - 1) // ALIGN * ALIGN
            self.groups.append([p for _, p in grp])
            for n, p in grp:
                self.local[id(p)] = off
                self.params.append(p)
                self.names.append(n)
                off += p.numel()
        self.numel = off
        chunk = ALIGN * self.world
        self.padded = max(chunk, (off + chunk - 1) // chunk * chunk)
        self.per = self.padded // self.world
        self.soff = 0      # offset of this rank's shard in the store's shard buffers
        self.voff = 0      # offset of the unit in the full (virtual) flat layout
        self.full: Optional[torch.Tensor] = None    # gathered weights, compute dtype
        self.gfull: Optional[torch.Tensor] = None   # full fp32 gradient
        self.state = _FREE
        self.work = None
        self.stale = True
        self.grad_live = False

    def src(self) -> int:
        """Global rank whose initial values every member starts from."""
        return dist.get_global_rank(self.group, 0) if self.group is not None else 0


class BlockUnits:
    """The units of one transformer block (its dense matrices; under expert
    parallelism also its local experts), gathered before the block and
    released after it in the forward and again in the backward."""

    def __init__(self, store: "FullyShardedStore", parts: List[ParamUnit]):
        self.store = store
        self.parts = parts
        self.persistent = all(u.persistent for u in parts)
        self.in_backward = False
        self.prev: Optional["BlockUnits"] = None
        self.next: Optional["BlockUnits"] = None

    def _gather(self, wait: bool = True) -> None:
        for u in self.parts:
            self.store.gather(u, wait=wait)

    def _release(self) -> None:
        for u in self.parts:
            if not u.persistent:
                self.store.release(u)

    def enter(self, resid: torch.Tensor, delta: Optional[torch.Tensor]):
        """Block pre-forward: gather, prefetch the next block, and arm the
        post-backward hook on the block's inputs."""
        st = self.store
        self._gather()
        if not self.in_backward and self.next is not None and not st.pinned:
            self.next._gather(wait=False)
        if torch.is_grad_enabled() and resid.requires_grad and not self.in_backward:
            if delta is not None and delta.requires_grad:
                resid, delta = _Hook.apply(self._post_backward, resid, delta)
            else:
                (resid,) = _Hook.apply(self._post_backward, resid)
        return resid, delta

    def leave(self, resid: torch.Tensor, out: torch.Tensor, aux: Optional[torch.Tensor] = None):
        """Block post-forward: arm the pre-backward hook on the outputs (an
        MoE block's auxiliary loss included: its gradient reaches the router
        weights without passing through the other outputs) and release the
        gathered weights (not while the backward recomputes a checkpointed
        block).  Returns (resid, out, aux)."""
        st = self.store
        if torch.is_grad_enabled() and resid.requires_grad and not self.in_backward:
            if aux is not None and aux.requires_grad:
                resid, out, aux = _Hook.apply(self._pre_backward, resid, out, aux)
            else:
                resid, out = _Hook.apply(self._pre_backward, resid, out)
        # the last block's weights are needed again at once by the backward
        keep = self.next is None and torch.is_grad_enabled() and resid.requires_grad
        if not self.in_backward and not st.pinned and not keep:
            self._release()
        return resid, out, aux

    def _pre_backward(self) -> None:
        self.in_backward = True
        self._gather()
        for u in self.parts:
            self.store.alloc_grad(u)
        if self.prev is not None:
            self.prev._gather(wait=False)

    def _post_backward(self) -> None:
        if not self.in_backward:
            return
        self.in_backward = False
        for u in self.parts:
            self.store.reduce_grad(u)
        if not self.store.pinned:
            self._release()


class _Hook(torch.autograd.Function):
    """Identity on its tensors whose backward first calls ``fn()`` (once,
    when the gradients of all of them are available)."""

    @staticmethod
    def forward(ctx, fn, *xs):
        ctx.fn = fn
        return tuple(x.view_as(x) for x in xs)

    @staticmethod
    def backward(ctx, *gs):
        ctx.fn()
        return (None,) + gs


class FullyShardedStore:
    """Parameter store with sharded weights / gradients (the interface the
    ops use: ``fused_view``, ``compute_of``, ``grad_of``; the optimizer's:
    ``master``, ``grad``, ``compute``, ``decay_end``, ``params``,
    ``offset``) and the data-parallel hooks the training engine calls
    (``begin_step``, ``finish_backward``, ``after_step``, ...)."""

    mode = "fsdp"

    def __init__(self, model: nn.Module, group=None, compute_dtype: Optional[torch.dtype] = None,
                 device: Optional[torch.device] = None, reshard_after_forward: bool = True,
                 expert_group=None, tp_group=None, local: bool = False):
        """``expert_group``: under expert parallelism, the ranks that hold the
        same experts (one per expert-parallel block); each block's local
        experts form a unit sharded over it.  ``tp_group``: under tensor
        parallelism the units hold this rank's tensor shards (sharded again
        over ``group``, the data-parallel ranks of the same tensor shard), and
        the gradients of replicated parameters that are partial per tensor
        rank (``_tp_reduce == "sum"``) are summed over ``tp_group`` before
        each unit's reduce-scatter.  ``local``: one data-parallel replica (no
        sharding of the dense units; ``group`` is ignored)."""
        self.model = model
        self.tp_group = tp_group if (tp_group is not None and is_dist()
                                     and get_world_size(tp_group) > 1) else None
        self.group = group
        self.world = 1 if local else get_world_size(group)
        self.rank = 0 if local else get_rank(group)
        dev = device or next(model.parameters()).device
        self.device = dev
        if compute_dtype is None:
            compute_dtype = torch.bfloat16 if dev.type == "cuda" else torch.float32
        self.compute_dtype = compute_dtype
        self.distributed = is_dist() and self.world > 1
        self.nccl = self.distributed and dist.get_backend(group) == "nccl"
        self.pinned = False
        self.final_micro = True

        blocks, per_block, per_block_experts, rest_decay, rest_nodecay, small = partition(model)
        # the expert gradient's data-parallel mean: summed over the ranks
        # holding the same experts, divided by the data-parallel world
        # (no group: every expert set exists once, on this rank)
        e_local = expert_group is None
        e_scale = (1 if e_local else get_world_size(expert_group)) / max(1, self.world)
        keep = not reshard_after_forward
        units: List[ParamUnit] = []
        self.blocks: List[BlockUnits] = []
        for bi in range(len(blocks)):
            parts = []
            if per_block[bi]:
                parts.append(ParamUnit(f"layers.{bi}", per_block[bi], compute_dtype, keep, True,
                                       group, local=local))
            if per_block_experts[bi]:
                parts.append(ParamUnit(f"layers.{bi}.experts", per_block_experts[bi], compute_dtype,
                                       keep, True, expert_group, grad_scale=e_scale,
                                       local=e_local))
            if not parts:
                continue
            units += parts
            sched = BlockUnits(self, parts)
            blocks[bi].param_unit = sched
            self.blocks.append(sched)
        for a, b in zip(self.blocks, self.blocks[1:]):
            a.next, b.prev = b, a
        self.block_units = [u for b in self.blocks for u in b.parts]
        if rest_decay:
            units.append(ParamUnit("root_decay", rest_decay, compute_dtype, True, True, group,
                                   local=local))
        if rest_nodecay:
            units.append(ParamUnit("root_nodecay", rest_nodecay, compute_dtype, True, False, group,
                                   local=local))
        if small:
            units.append(ParamUnit("fp32_1d", small, torch.float32, True, False, group,
                                   local=local))
        self.units = units
        for u in units:
            u.tp_sum = ([(u.local[id(p)], p.numel()) for p in u.params
                         if getattr(p, "_tp_reduce", "none") == "sum"]
                        if self.tp_group is not None else [])

        soff = voff = 0
        self.decay_end = 0
        for u in units:
            u.soff, u.voff = soff, voff
            soff += u.per
            voff += u.padded
            if u.decay:
                self.decay_end = soff
        self.shard_numel = soff
        self.numel = voff   # size of the full (virtual) layout
        self.master = torch.zeros(soff, dtype=torch.float32, device=dev)
        self.grad = torch.zeros(soff, dtype=torch.float32, device=dev)
        self.compute = (torch.zeros(soff, dtype=compute_dtype, device=dev)
                        if compute_dtype != torch.float32 else None)
        self.params: List[nn.Parameter] = [p for u in units for p in u.params]
        self.names: List[str] = [n for u in units for n in u.names]
        self.offsets: Dict[int, int] = {id(p): u.voff + u.local[id(p)] for u in units for p in u.params}
        self.unit_of: Dict[int, ParamUnit] = {id(p): u for u in units for p in u.params}
        self.fp32_span = (0, 0)
        self.expert_span = (0, 0)
        self.shard = (0, soff)
        self._pviews: Dict[int, torch.Tensor] = {}
        self._gviews: Dict[int, torch.Tensor] = {}
        self._fviews: Dict[tuple, Tuple[torch.Tensor, torch.Tensor]] = {}
        self._rs_stream = (torch.cuda.Stream(device=dev)
                           if any(u.nccl for u in units) else None)
        with torch.no_grad():
            for u in units:
                self._init_unit(u)
        model.param_store = self
        # the persistent units are gathered before the model runs: from
        # ``Qwen3Model.hidden`` (every forward path, direct calls included)
        # and from a pre-forward hook for other model classes
        model.param_gather = self.gather_root
        self._hook = model.register_forward_pre_hook(lambda m, a: self.gather_root())

    # ------------------------------------------------------------ set-up
    def _init_unit(self, u: ParamUnit) -> None:
        """Shard the unit's initial values (rank 0's, broadcast), build the
        gathered / gradient buffers and every view of them, then release
        the buffers."""
        dev = self.device
        tmp = torch.zeros(u.padded, dtype=torch.float32, device=dev)
        for p in u.params:
            o = u.local[id(p)]
            tmp[o:o + p.numel()].copy_(p.detach().reshape(-1).to(dev, torch.float32))
        if u.distributed:
            dist.broadcast(tmp, src=u.src(), group=u.group)
        mine = tmp[u.rank * u.per:(u.rank + 1) * u.per]
        self.master[u.soff:u.soff + u.per].copy_(mine)
        if self.compute is not None:
            self.compute[u.soff:u.soff + u.per].copy_(mine)
        u.full = torch.empty(u.padded, dtype=u.dtype, device=dev)
        u.gfull = torch.zeros(u.padded, dtype=torch.float32, device=dev)
        for p in u.params:
            o, n = u.local[id(p)], p.numel()
            self._pviews[id(p)] = u.full[o:o + n].view(p.shape)
            self._gviews[id(p)] = u.gfull[o:o + n].view(p.shape)
            if p.dim() >= 2:
                self._fviews[(id(p),)] = (u.full[o:o + n].view(-1, p.shape[-1]),
                                          u.gfull[o:o + n].view(-1, p.shape[-1]))
        for grp in u.groups:
            if len(grp) < 2 or any(p.dim() < 2 for p in grp):
                continue
            K = grp[0].shape[-1]
            o0 = u.local[id(grp[0])]
            o, ok = o0, True
            for p in grp:
                if u.local[id(p)] != o or p.shape[-1] != K:
                    ok = False
                    break
                o += p.numel()
            if ok:
                self._fviews[tuple(id(p) for p in grp)] = (u.full[o0:o].view(-1, K),
                                                           u.gfull[o0:o].view(-1, K))
        for p in u.params:
            p.data = self._pviews[id(p)]
            p.grad = None
            p._nq_store = self
            p._nq_offset = self.offsets[id(p)]
        # the initial values are sharded now: the gathered copy is filled on
        # first use
        _set_storage(u.full, 0)
        _set_storage(u.gfull, 0)
        u.state, u.stale, u.grad_live = _FREE, True, False

    # ------------------------------------------------------- views for ops
    def offset(self, p: torch.Tensor) -> int:
        return self.offsets[id(p)]

    def fused_view(self, params: Sequence[torch.Tensor], dtype: torch.dtype):
        """(gathered weights [N, K], fp32 gradient [N, K]) of ``cat(params)``
        or None (not a unit's contiguous group, or another dtype)."""
        key = tuple(id(p) for p in params)
        v = self._fviews.get(key)
        if v is None or v[0].dtype != dtype:
            return None
        u = self.unit_of[key[0]]
        if u.state != _READY:
            self.gather(u)
        return v

    def compute_of(self, p: torch.Tensor) -> torch.Tensor:
        u = self.unit_of[id(p)]
        if u.state != _READY:
            self.gather(u)
        return self._pviews[id(p)]

    def grad_of(self, p: torch.Tensor) -> torch.Tensor:
        u = self.unit_of[id(p)]
        if not u.grad_live:
            self.alloc_grad(u)
        return self._gviews[id(p)]

    def num_parameters(self) -> int:
        return sum(p.numel() for p in self.params)

    # ------------------------------------------------------------ gathers
    def _source(self, u: ParamUnit) -> torch.Tensor:
        buf = self.master if (u.dtype == torch.float32 or self.compute is None) else self.compute
        return buf[u.soff:u.soff + u.per]

    def gather(self, u: ParamUnit, wait: bool = True) -> None:
        """Make the unit's full weights available (``wait=False``: only
        issue the all-gather)."""
        if u.state == _READY and not u.stale:
            return
        if u.state == _GATHERING:
            if wait:
                self._wait(u)
            return
        _set_storage(u.full, u.padded)
        src = self._source(u)
        if not u.distributed:
            u.full.copy_(src)
            u.state = _READY
        elif u.nccl:
            u.work = dist.all_gather_into_tensor(u.full, src, group=u.group, async_op=True)
            u.state = _GATHERING
        else:
            all_gather_flat_(u.full, src, u.group)
            u.state = _READY
        u.stale = False
        if wait:
            self._wait(u)

    def _wait(self, u: ParamUnit) -> None:
        if u.work is not None:
            u.work.wait()
            u.work = None
        u.state = _READY

    def release(self, u: ParamUnit) -> None:
        if u.state == _FREE:
            return
        self._wait(u)
        _set_storage(u.full, 0)
        u.state = _FREE

    def gather_root(self) -> None:
        """Model pre-forward: the persistent units (embedding, lm_head, 1-D
        parameters) gathered, with gradient buffers when training."""
        for u in self.units:
            if u.persistent:
                self.gather(u)
                if torch.is_grad_enabled() and self.model.training and not u.grad_live:
                    self.alloc_grad(u)

    # ----------------------------------------------------------- gradients
    def alloc_grad(self, u: ParamUnit) -> None:
        """A zeroed fp32 gradient buffer for the unit.  Parameters of the
        same dtype (fp32: the 1-D unit, every unit on the CPU) also get it as
        ``.grad``, so autograd's own accumulation (norm weights, the CPU
        embedding) lands in the buffer in place."""
        if u.grad_live:
            return
        _set_storage(u.gfull, u.padded)
        u.gfull.zero_()
        u.grad_live = True
        for p in u.params:
            gv = self._gviews[id(p)]
            if gv.dtype == p.dtype:
                p.grad = gv

    def reduce_grad(self, u: ParamUnit) -> None:
        """Mean over ranks of the unit's gradient, added into this rank's
        gradient shard; the full gradient buffer is released."""
        if not u.grad_live:
            return
        g = self.grad[u.soff:u.soff + u.per]
        if not u.distributed:
            self._tp_sum(u)
            g.add_(u.gfull, alpha=u.grad_scale)
        elif u.nccl:
            side = self._rs_stream
            side.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(side):
                self._tp_sum(u)
                tmp = torch.empty(u.per, dtype=torch.float32, device=self.device)
                dist.reduce_scatter_tensor(tmp, u.gfull, op=dist.ReduceOp.AVG, group=u.group)
                g.add_(tmp, alpha=u.grad_scale)
            u.gfull.record_stream(side)
        else:
            self._tp_sum(u)
            tmp = torch.empty(u.per, dtype=torch.float32, device=self.device)
            reduce_scatter_avg_(tmp, u.gfull, u.group)
            g.add_(tmp, alpha=u.grad_scale)
        for p in u.params:
            p.grad = None
        _set_storage(u.gfull, 0)
        u.grad_live = False

    def _tp_sum(self, u: ParamUnit) -> None:
        """Sum the partial gradients of tensor-replicated parameters over the
        tensor-parallel group (one all-reduce per unit)."""
        if not u.tp_sum:
            return
        flat = torch.cat([u.gfull[o:o + n] for o, n in u.tp_sum])
        dist.all_reduce(flat, group=self.tp_group)
        k = 0
        for o, n in u.tp_sum:
            u.gfull[o:o + n].copy_(flat[k:k + n])
            k += n

    def shard_slices(self, p: torch.Tensor) -> List[Tuple[int, int]]:
        """Ranges of this rank's shard buffers that hold elements of ``p``."""
        u = self.unit_of[id(p)]
        v0 = u.local[id(p)]
        v1 = v0 + p.numel()
        a, b = u.rank * u.per, (u.rank + 1) * u.per
        lo, hi = max(v0, a), min(v1, b)
        return [(u.soff + lo - a, u.soff + hi - a)] if hi > lo else []

    # ------------------------------------------------- engine-facing hooks
    def begin_step(self, final_micro: bool) -> None:
        """Called before each micro-batch's forward."""
        self.final_micro = final_micro

    def finish_backward(self) -> None:
        """After a micro-batch's backward: reduce what no hook reduced (a
        block whose input needed no gradient) and, after the last
        micro-batch, the persistent units' accumulated gradients."""
        for b in self.blocks:
            if b.in_backward:
                b._post_backward()
            elif any(u.grad_live for u in b.parts):
                for u in b.parts:
                    self.reduce_grad(u)
                if not self.pinned:
                    b._release()
        if self.final_micro:
            for u in self.units:
                if u.persistent and u.grad_live:
                    self.reduce_grad(u)
        if self._rs_stream is not None:
            torch.cuda.current_stream(self.device).wait_stream(self._rs_stream)

    def sync_grads(self) -> None:
        """Gradients are already reduced into the shards by the hooks."""
        return

    def norm_sq_reduce(self, sq: torch.Tensor) -> torch.Tensor:
        if not self.distributed:
            return sq
        sq = sq.clone()
        dist.all_reduce(sq, group=self.group)
        return sq

    def after_step(self) -> None:
        """The optimizer rewrote the shards: every gathered copy is stale."""
        for u in self.units:
            u.stale = True

    def gather_params(self) -> None:
        self.after_step()

    def zero_grad(self) -> None:
        self.grad.zero_()

    def reattach_grads(self) -> None:
        return

    @torch.no_grad()
    def refresh_compute(self) -> None:
        """Recast the master shard into the compute shard (after a load)."""
        if self.compute is not None:
            self.compute.copy_(self.master)
        self.after_step()

    def broadcast_params(self, src: int = 0) -> None:
        """Rank 0's initial values were broadcast when the units were built."""
        return

    def gather_master(self) -> None:
        return

    @contextlib.contextmanager
    def summon_full_params(self):
        """Every unit gathered and kept (generation / evaluation inside a
        training run)."""
        prev = self.pinned
        self.pinned = True
        try:
            for u in self.units:
                self.gather(u)
            yield
        finally:
            self.pinned = prev
            if not prev:
                for b in self.blocks:
                    if not b.in_backward:
                        b._release()

    # --------------------------------------------- full (virtual) buffers
    @torch.no_grad()
    def gather_virtual(self, shard_buf: torch.Tensor) -> torch.Tensor:
        """A full-layout copy of a shard-layout fp32 buffer (master, a
        moment): unit u at [voff, voff + padded)."""
        out = torch.zeros(self.numel, dtype=shard_buf.dtype, device=shard_buf.device)
        for u in self.units:
            dst = out[u.voff:u.voff + u.padded]
            src = shard_buf[u.soff:u.soff + u.per].contiguous()
            if u.distributed:
                all_gather_flat_(dst, src, u.group)
            else:
                dst.copy_(src)
        return out

    @torch.no_grad()
    def scatter_virtual(self, full: torch.Tensor, shard_buf: torch.Tensor) -> None:
        """This rank's part of a full-layout buffer back into shard layout."""
        for u in self.units:
            a = u.voff + u.rank * u.per
            shard_buf[u.soff:u.soff + u.per].copy_(full[a:a + u.per])

    def bind_full(self, full: torch.Tensor) -> None:
        """Parameters become views of a full-layout fp32 buffer."""
        for p in self.params:
            o = self.offsets[id(p)]
            p.data = full[o:o + p.numel()].view(p.shape)

    def bind_compute(self) -> None:
        """Parameters become views of their units' gathered buffers again."""
        for p in self.params:
            p.data = self._pviews[id(p)]

    def memory_bytes(self) -> Dict[str, int]:
        """Bytes this rank holds for weights / gradients between steps
        (optimizer moments excluded) and the largest transient unit."""
        el = self.compute.element_size() if self.compute is not None else 0
        shard = self.shard_numel * (4 + 4 + el)
        persistent = sum(u.padded * (u.full.element_size() + 4) for u in self.units if u.persistent)
        largest = max((u.padded * (u.full.element_size() + 4) for u in self.block_units), default=0)
        return {"shards": shard, "persistent_units": persistent, "largest_block_unit": largest}


def memory_plan(model: nn.Module, world: int, compute_bytes: int = 2, ep: int = 1) -> Dict[str, float]:
    """Bytes per rank of ``model`` (a meta-device model will do: nothing is
    allocated) fully sharded over ``world`` ranks, next to the flat ZeRO-2
    layout of ``FlatParamStore`` + ``FusedAdamW``:

    * ``fsdp_state``: the shards (fp32 master and gradient, the compute copy
      and the two fp32 Adam moments, 18 B per element with bf16);
    * ``fsdp_persistent``: embedding / lm_head / 1-D units, gathered for a
      step with their fp32 gradients;
    * ``fsdp_blocks_peak``: two gathered block units (the running block and
      the prefetched one) and one block's fp32 gradient;
    * ``zero2_state``: full fp32 master, gradient and compute copy on every
      rank, moments sharded;
    * with ``ep`` > 1 (``model`` holding every expert, ``.experts.`` in their
      names): ``zero2_ep_state``, the ZeRO-2 state of one rank that holds
      1/ep of the experts, its expert moments sharded over the world / ep
      ranks holding the same experts, and ``zero2_ep_replicated_state``, the
      same with every moment of the rank's parameters kept (what replicating
      the gradients of expert-parallel runs costs)."""
    _, pb, pbe, rd, rn, small = partition(model)
    units = []
    for gs in pb + pbe:
        if gs:
            units.append(("block", ParamUnit("b", gs, torch.bfloat16, False, True, world=world)))
    for kind, gs, fp32 in (("root", rd, False), ("root", rn, False), ("root", small, True)):
        if gs:
            units.append((kind, ParamUnit(kind, gs, torch.float32 if fp32 else torch.bfloat16, True,
                                          True, world=world)))
    shard = sum(u.per for _, u in units)
    state = shard * (4 + 4 + compute_bytes + 8)
    persistent = sum(u.padded * ((4 if u.dtype == torch.float32 else compute_bytes) + 4)
                     for k, u in units if k == "root")
    biggest = max((u.padded for k, u in units if k == "block"), default=0)
    peak_blocks = biggest * (2 * compute_bytes + 4)
    numel = sum(p.numel() for p in model.parameters() if p.requires_grad)
    zero2 = numel * (4 + 4 + compute_bytes) + numel * 8 / world
    out = {"params": float(numel), "fsdp_state": float(state), "fsdp_persistent": float(persistent),
           "fsdp_blocks_peak": float(peak_blocks),
           "fsdp_total": float(state + persistent + peak_blocks), "zero2_state": float(zero2)}
    if ep > 1:
        expert = sum(p.numel() for n, p in model.named_parameters()
                     if p.requires_grad and ".experts." in n)
        dense, local = numel - expert, expert / ep
        resident = (dense + local) * (4 + 4 + compute_bytes)
        out["zero2_ep_state"] = float(resident + dense * 8 / world + local * 8 / (world / ep))
        out["zero2_ep_replicated_state"] = float(resident + (dense + local) * 8)
    return out


class FSDPAdamW(FusedAdamW):
    """AdamW over a ``FullyShardedStore``: the moments have the shard's
    size, the step is the fused AdamW kernel over the shard buffers (it
    also writes the compute shard the next all-gathers read), and
    ``gather_full_state`` exposes full fp32 parameters and moments under
    the single-process names for a checkpoint save or load."""

    # ``gather_full_state`` rebinds the parameters (checkpoint saves of this
    # optimizer run synchronously)
    full_state_rebinds_params = True

    def __init__(self, store: FullyShardedStore, lr: float = 3e-4, betas=(0.9, 0.95),
                 eps: float = 1e-8, weight_decay: float = 0.1):
        self.store = store
        decay = [p for u in store.units if u.decay for p in u.params]
        nodecay = [p for u in store.units if not u.decay for p in u.params]
        groups = []
        if decay:
            groups.append({"params": decay, "weight_decay": weight_decay})
        if nodecay:
            groups.append({"params": nodecay, "weight_decay": 0.0})
        torch.optim.Optimizer.__init__(self, groups, dict(lr=lr, betas=betas, eps=eps,
                                                          weight_decay=weight_decay))
        dev = store.master.device
        n = store.shard_numel
        self.shard = (0, n)
        self.sharded = True
        self.state_base = 0
        self.exp_avg = torch.zeros(n, dtype=torch.float32, device=dev)
        self.exp_avg_sq = torch.zeros(n, dtype=torch.float32, device=dev)
        self._full = None
        self._full_params = None
        self.state_gather = None
        self.step_count = 0
        self.clip_scale = torch.ones((), dtype=torch.float32, device=dev)
        self.last_grad_norm = torch.zeros((), dtype=torch.float32, device=dev)
        for p in store.params:
            self.state[p] = {"step": torch.zeros((), dtype=torch.float32)}

    @torch.no_grad()
    def clip_grad_norm_(self, max_norm: float, norm_sq_reduce=None) -> torch.Tensor:
        self.store.finish_backward()
        return super().clip_grad_norm_(max_norm, norm_sq_reduce or self.store.norm_sq_reduce)

    @torch.no_grad()
    def step(self, closure=None, update=None):
        # gradients still in full buffers (a loop without the training
        # engine's per-micro-batch hook) are reduced into the shards first
        self.store.finish_backward()
        out = super().step(closure, update)
        self.store.after_step()
        return out

    @torch.no_grad()
    def gather_full_state(self, gather=None) -> None:
        if self._full is not None:
            return
        st = self.store
        m = st.gather_virtual(self.exp_avg)
        v = st.gather_virtual(self.exp_avg_sq)
        self._full_params = st.gather_virtual(st.master)
        st.bind_full(self._full_params)
        self._full = [m, v]
        self._bind_views(m, v)

    @torch.no_grad()
    def release_full_state(self, scatter: bool = False) -> None:
        if self._full is None:
            return
        st = self.store
        if scatter:
            st.scatter_virtual(self._full[0], self.exp_avg)
            st.scatter_virtual(self._full[1], self.exp_avg_sq)
            st.scatter_virtual(self._full_params, st.master)
            st.refresh_compute()
        st.bind_compute()
        for p in st.params:
            self.state[p].pop("exp_avg", None)
            self.state[p].pop("exp_avg_sq", None)
        self._full = None
        self._full_params = None



def build_fsdp_optimizer(store: FullyShardedStore, lr: float = 3e-4, weight_decay: float = 0.1,
                         beta1: float = 0.9, beta2: float = 0.95, eps: float = 1e-8):
    return FSDPAdamW(store, lr=lr, betas=(beta1, beta2), eps=eps, weight_decay=weight_decay)


# ---------------------------------------------------------------- reference API
class MixedPrecisionPolicy:
    """Gathered-parameter dtype and gradient-reduction dtype (the fields of
    FSDP2's policy; reference: distributed/fsdp.py:36-41)."""

    def __init__(self, param_dtype: torch.dtype = torch.bfloat16,
                 reduce_dtype: torch.dtype = torch.float32):
        self.param_dtype = param_dtype
        self.reduce_dtype = reduce_dtype


def get_mixed_precision_policy(dtype: str = "bfloat16") -> MixedPrecisionPolicy:
    return MixedPrecisionPolicy(param_dtype=getattr(torch, dtype, torch.bfloat16),
                                reduce_dtype=torch.float32)


def apply_fsdp2(model: nn.Module, mesh=None, mp_policy: Optional[MixedPrecisionPolicy] = None,
                reshard_after_forward: bool = True) -> nn.Module:
    """Shard ``model`` per transformer block plus a root unit (the call the
    reference makes, reference: distributed/fsdp.py:44-75).  ``mesh``: a
    process group, a 1-D ``DeviceMesh`` or None (the default group).  The
    gathered weights use ``mp_policy.param_dtype`` on the GPU; gradients are
    reduced in fp32.  ``build_optimizer(model)`` then returns ``FSDPAdamW``."""
    group = mesh.get_group() if hasattr(mesh, "get_group") else mesh
    dev = next(model.parameters()).device
    dtype = None
    if mp_policy is not None and dev.type == "cuda":
        dtype = mp_policy.param_dtype
    FullyShardedStore(model, group=group, compute_dtype=dtype,
                      reshard_after_forward=reshard_after_forward)
    return model


def apply_fsdp1(model: nn.Module, dtype: str = "bfloat16", cpu_offload: bool = False,
                sharding_strategy: str = "FULL_SHARD") -> nn.Module:
    """The reference's FSDP1 fallback (reference: distributed/fsdp.py:78-101)
    maps to the same sharding; CPU offload is not provided (180 GB of HBM per
    GPU holds the shards of every configuration here)."""
    if cpu_offload:
        raise NotImplementedError("CPU offload of parameter shards")
    if sharding_strategy not in ("FULL_SHARD", "SHARD_GRAD_OP"):
        raise ValueError(f"sharding strategy {sharding_strategy!r}")
    return apply_fsdp2(model, None, get_mixed_precision_policy(dtype),
                       reshard_after_forward=sharding_strategy == "FULL_SHARD")
