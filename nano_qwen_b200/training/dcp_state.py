"""Layout-independent DCP state for model-parallel runs.

Under tensor, expert or pipeline parallelism a rank holds pieces of the
logical model: row or column shards of the TP linears, a contiguous block of
experts, a contiguous block of layers.  The reference saves whatever sharding
it runs through torch.distributed.checkpoint with the full model's names
(reference: training/checkpoint.py:104-141); this module gives the same
property to this library's layouts, so a checkpoint written at one layout
loads at another (tp2 -> tp1, ep2 -> ep1, pp2 -> pp1 and back):

* every parameter gets its *logical* name: local layer indices shifted by the
  pipeline stage's first layer, local expert indices shifted by the rank's
  first expert (``layers.3.ffn.experts.17.ffn.down_proj.weight``), the names
  the single-process ``Qwen3Model`` uses;
* a TP shard becomes a ``DTensor`` over the TP group with its ``Shard(dim)``
  placement and the full logical shape, so DCP writes chunks at their global
  offsets and reads back whichever chunks another layout asks for;
* everything else is a plain tensor (replicated ranks write it once).

The Adam moments follow their parameter (same name, placement and shape
under ``optimizer.state.<name>.exp_avg`` / ``exp_avg_sq`` / ``step``).
"""

from __future__ import annotations

import re
from typing import Dict, List, Optional, Tuple

import torch
import torch.nn as nn

_LAYER = re.compile(r"^layers\.(\d+)\.")
_EXPERT = re.compile(r"\.experts\.(\d+)\.")


def _base(model: nn.Module) -> Tuple[nn.Module, int]:
    """(module whose parameter names are Qwen3Model's, first global layer)."""
    if hasattr(model, "layer_offset") and hasattr(model, "model"):  # PipelineParallel
        return model.model, int(model.layer_offset)
    return model, 0


def _expert_offsets(base: nn.Module) -> Dict[int, int]:
    out = {}
    for m in base.modules():
        off = getattr(m, "expert_offset", None)
        if off and hasattr(m, "experts"):
            for p in m.experts.parameters():
                out[id(p)] = int(off)
    return out


def _tp_dims(base: nn.Module) -> Dict[int, Tuple[int, object]]:
    """id(param) -> (shard dim, TP group) for the sharded linears."""
    out = {}
    for m in base.modules():
        mode = getattr(m, "tp_mode", None)
        if mode is None:
            continue
        grp = m.tp_group
        if getattr(m.weight, "_tp_sharded", False):
            out[id(m.weight)] = (0 if mode == "col" else 1, grp)
        b = getattr(m, "bias", None)
        if b is not None and getattr(b, "_tp_sharded", False):
            out[id(b)] = (0, grp)
    return out


def logical_name(name: str, layer_off: int, expert_off: int) -> str:
    if layer_off:
        name = _LAYER.sub(lambda mt: f"layers.{int(mt.group(1)) + layer_off}.", name, count=1)
    if expert_off:
        name = _EXPERT.sub(lambda mt: f".experts.{int(mt.group(1)) + expert_off}.", name, count=1)
    return name


def logical_params(model: nn.Module) -> List[Tuple[str, nn.Parameter, Optional[Tuple[int, object]], bool]]:
    """(logical name, local parameter, (shard dim, TP group) or None, alias):
    ``alias`` marks a second name of an already listed tensor (a tied
    lm_head), which has model state but no optimizer state of its own."""
    base, layer_off = _base(model)
    experts = _expert_offsets(base)
    tp = _tp_dims(base)
    out = []
    seen = set()
    for n, p in base.named_parameters():
        if id(p) in seen:
            continue
        seen.add(id(p))
        out.append((logical_name(n, layer_off, experts.get(id(p), 0)), p, tp.get(id(p)), False))
    # a tied lm_head shares the embedding's tensor: the single-process model's
    # state dict lists it under both names, so write it under both too
    if getattr(base, "lm_head", None) is not None and getattr(base, "embed", None) is not None:
        w = base.lm_head.weight
        if w is base.embed.embed_tokens.weight:
            out.append(("lm_head.weight", w, None, True))
    return out


def _mesh(group, device_type: str):
    from torch.distributed.device_mesh import DeviceMesh
    key = (id(group), device_type)
    cache = _mesh.__dict__.setdefault("cache", {})
    if key not in cache:
        cache[key] = DeviceMesh.from_group(group, device_type)
    return cache[key]


def _wrap(t: torch.Tensor, shard) -> torch.Tensor:
    """A TP shard as a DTensor with the full logical shape."""
    if shard is None:
        return t
    import torch.distributed as dist
    from torch.distributed.tensor import DTensor, Shard
    dim, grp = shard
    ws = dist.get_world_size(grp)
    shape = list(t.shape)
    shape[dim] *= ws
    stride = torch.empty(shape, device="meta").stride()
    return DTensor.from_local(t, _mesh(grp, t.device.type), [Shard(dim)], run_check=False,
                              shape=torch.Size(shape), stride=stride)


def model_parallel_state(model: nn.Module, optimizer=None) -> dict:
    """The DCP state of a model-parallel run: ``model.<logical name>`` and
    ``optimizer.state.<logical name>.{exp_avg, exp_avg_sq, step}``.  Tensors
    are the live parameters / moment views (DCP reads them on save and writes
    into them on load)."""
    sd: dict = {"model": {}}
    ost: dict = {}
    for name, p, shard, alias in logical_params(model):
        sd["model"][name] = _wrap(p.data, shard)
        if optimizer is not None and not alias and p in optimizer.state:
            st = optimizer.state[p]
            entry = {}
            for k in ("exp_avg", "exp_avg_sq"):
                if k in st:
                    entry[k] = _wrap(st[k], shard)
            if "step" in st:
                entry["step"] = st["step"]
            if entry:
                ost[name] = entry
    if optimizer is not None:
        sd["optimizer"] = {"state": ost}
    return sd


def logical_load_state(model: nn.Module, optimizer=None) -> dict:
    """Load targets for any run, model-parallel or not: the same keys as
    ``model_parallel_state`` (the single-process names), so a checkpoint of
    one layout loads into another.  Optimizer moments must be bound (a
    sharded optimizer calls ``gather_full_state`` first)."""
    return model_parallel_state(model, optimizer)
