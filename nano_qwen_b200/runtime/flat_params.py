"""Flat parameter / gradient / compute-copy storage.

All trainable parameters of a model are re-homed into three flat device
buffers: fp32 master weights, fp32 gradients and (on GPU) a bf16 compute copy.
Each ``nn.Parameter`` becomes a view of the master buffer, so module code,
``state_dict`` and torch.distributed.checkpoint see the usual names and shapes
(the reference's checkpoint keys, e.g. ``layers.0.attention.q_proj.weight``).

Layout rules:

* fusion groups declared by modules (q|k|v, gate|up, every expert's gate|up,
  every expert's down) are contiguous, so one GEMM sees one [N, K] view;
* weight-decay groups are contiguous: all decay tensors form one region
  [decay_begin, decay_end), which lets the fused AdamW kernel run over the
  whole store in one launch with the reference's grouping rule
  (reference: training/optimizer.py:36-45);
* group starts are 64-element aligned (16-byte TMA and vector alignment).

Data-parallel gradient buckets and ZeRO shards are plain slices of these
buffers, so collectives run on them without packing copies.
"""

from __future__ import annotations

from typing import Dict, List, Optional, Sequence, Tuple

import torch
import torch.nn as nn

ALIGN = 64


def no_decay_rule(name: str, p: torch.Tensor) -> bool:
    """The reference's no-decay rule (training/optimizer.py:40-43); a
    parameter may also be marked ``_no_decay`` (the last pipeline stage's
    copy of a tied embedding)."""
    return (p.ndim <= 1 or "norm" in name or "bias" in name or "embed" in name
            or bool(getattr(p, "_no_decay", False)))


def default_groups(model: nn.Module) -> List[List[Tuple[str, nn.Parameter]]]:
    """Fusion groups: modules may define ``fusion_groups()`` returning lists of
    parameter-name lists (relative to the module).  Everything else is a group
    of one, in ``named_parameters`` order."""
    named = dict(model.named_parameters())
    claimed = set()
    groups: List[List[Tuple[str, nn.Parameter]]] = []
    for mod_name, mod in model.named_modules():
        fg = getattr(mod, "fusion_groups", None)
        if fg is None:
            continue
        for grp in fg():
            full = [(f"{mod_name}.{n}" if mod_name else n) for n in grp]
            items = [(n, named[n]) for n in full if n in named and id(named[n]) not in claimed]
            if len(items) != len(full):
                continue
            groups.append(items)
            claimed.update(id(p) for _, p in items)
    for n, p in model.named_parameters():
        if id(p) not in claimed:
            groups.append([(n, p)])
            claimed.add(id(p))
    # module order: each transformer block's weights end up contiguous, so a
    # block's gradients form one span that can be reduced as soon as the
    # block's backward is done
    order = {id(p): i for i, (_, p) in enumerate(model.named_parameters())}
    groups.sort(key=lambda g: order.get(id(g[0][1]), 0))
    return groups


class FlatParamStore:
    def __init__(self, model: nn.Module, compute_dtype: torch.dtype = torch.bfloat16,
                 device: Optional[torch.device] = None, trainable_only: bool = True,
                 pad_multiple: int = ALIGN, alloc=None):
        """``alloc(numel, dtype, device)`` (optional) allocates the gradient and
        compute-copy buffers, e.g. in peer-mapped symmetric memory for the
        peer-memory data-parallel step; it must return zero-filled tensors."""
        self.model = model
        self.compute_dtype = compute_dtype
        groups = default_groups(model)
        if trainable_only:
            groups = [g for g in groups if all(p.requires_grad for _, p in g)]
        decay = [g for g in groups if not no_decay_rule(g[0][0], g[0][1])]
        nodecay = [g for g in groups if no_decay_rule(g[0][0], g[0][1])]
        # Expert-parallel-local parameters (different experts on every EP rank)
        # form one contiguous span at the end of the decay region, so data
        # parallelism can reduce them over their own group.
        dense_decay = [g for g in decay if not getattr(g[0][1], "_ep_local", False)]
        expert_decay = [g for g in decay if getattr(g[0][1], "_ep_local", False)]
        decay = dense_decay + expert_decay
        ordered = decay + nodecay
        dev = device or next(model.parameters()).device
        self.device = dev
        offsets: Dict[int, int] = {}
        self.names: List[str] = []
        self.params: List[nn.Parameter] = []
        off = 0
        self.decay_begin = 0
        self.decay_end = 0
        self.group_spans: List[Tuple[int, int]] = []
        self.expert_span = (0, 0)
        # the expert span starts and ends on a multiple of pad_multiple (ALIGN
        # x the data-parallel world), so the dense pieces before and after it
        # and the span itself each split into equal shards
        span_pad = max(ALIGN, int(pad_multiple))
        for gi, grp in enumerate(ordered):
            off = (off + ALIGN - 1) // ALIGN * ALIGN
            if gi == len(dense_decay) and expert_decay:
                off = (off + span_pad - 1) // span_pad * span_pad
                self.expert_span = (off, 0)
            if gi == len(decay):
                if expert_decay:
                    off = (off + span_pad - 1) // span_pad * span_pad
                    self.expert_span = (self.expert_span[0], off)
                self.decay_end = off
            g0 = off
            for n, p in grp:
                offsets[id(p)] = off
                self.names.append(n)
                self.params.append(p)
                off += p.numel()
            self.group_spans.append((g0, off))
        if len(decay) == len(ordered):
            if expert_decay:
                off = (off + span_pad - 1) // span_pad * span_pad
                self.expert_span = (self.expert_span[0], off)
            self.decay_end = off
        # Padding to a multiple of (ALIGN * data-parallel world) lets reduce-scatter and
        # all-gather run on equal-size shards of the buffers themselves.
        pad = max(ALIGN, int(pad_multiple))
        self.numel = (off + pad - 1) // pad * pad
        self.master = torch.zeros(self.numel, dtype=torch.float32, device=dev)
        mk = alloc or (lambda n, dt, d: torch.zeros(n, dtype=dt, device=d))
        self.grad = mk(self.numel, torch.float32, dev)
        self.compute = mk(self.numel, compute_dtype, dev) if compute_dtype != torch.float32 else None
        self.offsets = offsets
        # Parameters that kernels read in fp32 from the master copy (norm
        # weights, biases: every 1-D parameter).  After a sharded optimizer step
        # this span of the master is re-synchronised across data-parallel ranks.
        one_d = [p for p in self.params if p.ndim <= 1]
        if one_d:
            lo = min(offsets[id(p)] for p in one_d)
            hi = max(offsets[id(p)] + p.numel() for p in one_d)
            if any(p.ndim > 1 and lo <= offsets[id(p)] < hi for p in self.params):
                lo, hi = self.decay_end, off
            self.fp32_span = (lo // ALIGN * ALIGN, min(self.numel, (hi + ALIGN - 1) // ALIGN * ALIGN))
        else:
            self.fp32_span = (0, 0)
        with torch.no_grad():
            for p in self.params:
                o = offsets[id(p)]
                view = self.master[o:o + p.numel()].view(p.shape)
                view.copy_(p.detach().to(dev, torch.float32))
                p.data = view
                p.grad = self.grad[o:o + p.numel()].view(p.shape)
                p._nq_store = self
                p._nq_offset = o
        self.refresh_compute()

    # ------------------------------------------------------------------ views
    def offset(self, p: torch.Tensor) -> int:
        return self.offsets[id(p)]

    def fused_view(self, params: Sequence[torch.Tensor], dtype: torch.dtype):
        """(compute [N,K], grad [N,K]) views of ``cat(params, 0)`` or None."""
        o0 = self.offsets.get(id(params[0]))
        if o0 is None:
            return None
        K = params[0].shape[-1] if params[0].dim() >= 2 else 1
        o = o0
        rows = 0
        for p in params:
            if self.offsets.get(id(p)) != o or p.dim() < 2 or p.shape[-1] != K:
                return None
            o += p.numel()
            rows += p.numel() // K
        n = o - o0
        if dtype == torch.float32 or self.compute is None:
            comp = self.master[o0:o0 + n].view(rows, K)
        elif dtype == self.compute_dtype:
            comp = self.compute[o0:o0 + n].view(rows, K)
        else:
            return None
        return comp, self.grad[o0:o0 + n].view(rows, K)

    def compute_of(self, p: torch.Tensor) -> torch.Tensor:
        o = self.offsets[id(p)]
        src = self.compute if self.compute is not None else self.master
        return src[o:o + p.numel()].view(p.shape)

    # ---------------------------------------------------------------- updates
    @torch.no_grad()
    def refresh_compute(self) -> None:
        """Recast the master weights into the compute copy (after loading)."""
        if self.compute is not None:
            self.compute.copy_(self.master)

    @torch.no_grad()
    def zero_grad(self) -> None:
        self.grad.zero_()

    def reattach_grads(self) -> None:
        """Restore the .grad views (e.g. after an optimizer set them to None)."""
        for p in self.params:
            o = self.offsets[id(p)]
            p.grad = self.grad[o:o + p.numel()].view(p.shape)

    def num_parameters(self) -> int:
        return sum(p.numel() for p in self.params)
