"""Checkpointing in the reference's on-disk format, with real resume state.

Layout (reference: training/checkpoint.py:37-189): ``save_dir/step_{step:08d}/``
holding a torch.distributed.checkpoint (DCP) save of ``{"model", "optimizer"}``
plus a rank-0 ``meta.json`` ``{step, scheduler, extra, ...}``; the plain
single-file fallback is ``checkpoint.pt`` ``{model, step, optimizer,
scheduler, extra}``, which is what ``train.py eval`` loads.  The newest
``max_checkpoints`` directories are kept.

Additions over the reference: the full CPU/CUDA RNG state and sampler state are
saved and restored (the reference saves 8 bytes of CPU RNG and never restores
them), ``async_save`` really runs DCP's ``async_save`` and the plain path keeps
``step`` on resume (reference: training/checkpoint.py:174 loses it).
Model-parallel runs (tensor / expert / pipeline shards) save through DCP
as well, under the single-process model's parameter names with TP shards as
DTensors (``dcp_state``), so a checkpoint of one layout loads into another;
their optimizer hyper-parameters go to ``meta.json``.  Loading always asks
DCP for the logical names, which also reads replicated and reference-written
checkpoints.
"""

from __future__ import annotations

import json
import shutil
from pathlib import Path
from typing import Any, Dict, Optional

import torch
import torch.nn as nn

from ..parallel.comm import barrier, get_rank, is_main_process

try:
    import torch.distributed.checkpoint as dcp
    from torch.distributed.checkpoint.state_dict import (get_model_state_dict,
                                                         get_optimizer_state_dict)
    HAS_DCP = True
except ImportError:  # pragma: no cover
    HAS_DCP = False


def _rng_state() -> Dict[str, Any]:
    st = {"cpu": torch.random.get_rng_state().tolist()}
    if torch.cuda.is_available():
        st["cuda"] = [s.tolist() for s in torch.cuda.get_rng_state_all()]
    return st


def _set_rng_state(st: Dict[str, Any]) -> None:
    if "cpu" in st:
        torch.random.set_rng_state(torch.tensor(st["cpu"], dtype=torch.uint8))
    if "cuda" in st and torch.cuda.is_available():
        states = [torch.tensor(s, dtype=torch.uint8) for s in st["cuda"]]
        if len(states) == torch.cuda.device_count():
            torch.cuda.set_rng_state_all(states)


def model_parallel(model: nn.Module) -> bool:
    """True when the parameters on this rank are shards (TP / EP) or a
    pipeline stage, so a replicated checkpoint format does not apply."""
    if hasattr(model, "pipeline_forward_backward"):
        return True
    return any(getattr(p, "_tp_sharded", False) or getattr(p, "_ep_local", False)
               for p in model.parameters())


def manager_from_config(training_config: dict, default_dir: str = "checkpoints") -> "CheckpointManager":
    """The checkpoint manager a training YAML's ``checkpoint`` section asks for."""
    ck = training_config.get("checkpoint", {}) or {}
    return CheckpointManager(save_dir=ck.get("save_dir", default_dir),
                             save_interval=ck.get("save_interval", 1000),
                             max_checkpoints=ck.get("max_checkpoints", 5),
                             async_save=ck.get("async_save", True))


def resolve_resume(resume_from: Optional[str], training_config: dict,
                   manager: Optional["CheckpointManager"] = None) -> Optional[str]:
    """The checkpoint directory (or file) to resume from: the command line's
    value, else the training YAML's ``checkpoint.resume_from`` (which the
    reference reads but never uses); ``latest`` / ``auto`` mean the newest
    ``step_*`` directory under the manager's save directory (None when there
    is none yet, i.e. a fresh start)."""
    value = resume_from or ((training_config.get("checkpoint", {}) or {}).get("resume_from"))
    if value in (None, "", "none", "null"):
        return None
    if str(value).lower() in ("latest", "auto"):
        return manager.latest() if manager is not None else None
    return str(value)


class CheckpointManager:
    def __init__(self, save_dir: str = "checkpoints", save_interval: int = 1000,
                 max_checkpoints: int = 5, async_save: bool = True, use_dcp: bool = True):
        self.save_dir = Path(save_dir)
        self.save_interval = save_interval
        self.max_checkpoints = max_checkpoints
        self.async_save = async_save
        self.use_dcp = use_dcp and HAS_DCP
        self._pending = None
        if is_main_process():
            self.save_dir.mkdir(parents=True, exist_ok=True)

    def should_save(self, step: int) -> bool:
        return step > 0 and self.save_interval > 0 and step % self.save_interval == 0

    # ------------------------------------------------------------------ save
    def save(self, step: int, model: nn.Module, optimizer=None, scheduler=None,
             extra_state: Optional[Dict[str, Any]] = None, sampler=None) -> Path:
        d = self.save_dir / f"step_{step:08d}"
        self.wait()
        # a sharded optimizer exposes full-shape moments only while a save or
        # load runs (gathered by the engine's state_for_save, or here)
        self._release = getattr(optimizer, "release_full_state", None)
        if self._release is not None:
            optimizer.gather_full_state()
        # a fully sharded optimizer points the parameters themselves at the
        # gathered tensors while they are saved, so its saves complete before
        # training resumes (no background write of tensors in use)
        self._async_now = self.async_save and not getattr(optimizer, "full_state_rebinds_params",
                                                          False)
        groups = None
        if optimizer is not None:
            groups = [{k: v for k, v in g.items() if k != "params" and isinstance(v, (int, float, list, tuple))}
                      for g in optimizer.param_groups]
        if model_parallel(model) and HAS_DCP:
            self._save_logical(d, model, optimizer)
        elif self.use_dcp:
            self._save_dcp(d, model, optimizer)
        else:
            self._save_plain(d, model, optimizer, scheduler, extra_state, step)
        if is_main_process():
            d.mkdir(parents=True, exist_ok=True)
            meta = {
                "step": step,
                "scheduler": scheduler.state_dict() if scheduler is not None else None,
                "extra": extra_state or {},
                "rng": _rng_state(),
                "sampler": sampler.state_dict() if sampler is not None else None,
            }
            if groups is not None:
                meta["optimizer_param_groups"] = groups
            with open(d / "meta.json", "w") as f:
                json.dump(meta, f)
            self._cleanup()
        if self._pending is None:
            self._release_full()
        barrier()
        return d

    def _release_full(self) -> None:
        rel, self._release = getattr(self, "_release", None), None
        if rel is not None:
            rel()

    def _save_logical(self, d: Path, model, optimizer):
        """Model-parallel runs: DCP save of the logical (single-process) state
        (the optimizer's hyper-parameters go to ``meta.json``)."""
        from .dcp_state import model_parallel_state
        sd = model_parallel_state(model, optimizer)
        if self._async_now and torch.distributed.is_initialized():
            self._pending = dcp.async_save(sd, checkpoint_id=str(d))
        else:
            dcp.save(sd, checkpoint_id=str(d))

    def _save_dcp(self, d: Path, model, optimizer):
        sd = {"model": get_model_state_dict(model)}
        if optimizer is not None:
            sd["optimizer"] = get_optimizer_state_dict(model, optimizer)
        if self._async_now and torch.distributed.is_initialized():
            self._pending = dcp.async_save(sd, checkpoint_id=str(d))
        else:
            dcp.save(sd, checkpoint_id=str(d))

    def _save_plain(self, d, model, optimizer, scheduler, extra, step):
        if not is_main_process():
            return
        d.mkdir(parents=True, exist_ok=True)
        state = {"model": model.state_dict(), "step": step}
        if optimizer is not None:
            state["optimizer"] = optimizer.state_dict()
        if scheduler is not None:
            state["scheduler"] = scheduler.state_dict()
        state["extra"] = dict(extra or {}, step=step)
        torch.save(state, d / "checkpoint.pt")

    def export_plain(self, path: str, model: nn.Module, step: int = 0) -> None:
        """Single-file ``checkpoint.pt`` (full state dict) for ``train.py eval``."""
        sd = get_model_state_dict(model) if HAS_DCP else model.state_dict()
        if is_main_process():
            torch.save({"model": {k: v.detach().cpu() for k, v in sd.items()}, "step": step}, path)

    def wait(self) -> None:
        if self._pending is not None:
            self._pending.result()
            self._pending = None
        self._release_full()

    # ------------------------------------------------------------------ load
    def load(self, model: nn.Module, optimizer=None, scheduler=None,
             checkpoint_dir: Optional[str] = None, sampler=None) -> Dict[str, Any]:
        self.wait()
        if checkpoint_dir is None:
            checkpoint_dir = self.latest()
            if checkpoint_dir is None:
                return {}
        d = Path(checkpoint_dir)
        shard = d / f"shard_{get_rank():05d}.pt"
        # full-shape parameters / moments to load into while the file is read
        # (a fully sharded store binds its parameters to full fp32 tensors)
        full = getattr(optimizer, "gather_full_state", None)
        if shard.exists():
            st = torch.load(shard, map_location="cpu", weights_only=False)
            if full is not None:
                full()
            try:
                model.load_state_dict(st["model"])
                if optimizer is not None and "optimizer" in st:
                    optimizer.load_state_dict(st["optimizer"])
            finally:
                if full is not None:
                    optimizer.release_full_state(scatter=True)
            out = {}
        elif (d / "checkpoint.pt").exists() and not (d / ".metadata").exists():
            if full is not None:
                full()
            try:
                out = self._load_plain(d, model, optimizer, scheduler)
            finally:
                if full is not None:
                    optimizer.release_full_state(scatter=True)
        else:
            self._load_logical(d, model, optimizer)
            out = {}
        store = getattr(model, "param_store", None)
        if store is not None:
            store.refresh_compute()
        meta_p = d / "meta.json"
        if meta_p.exists():
            with open(meta_p) as f:
                meta = json.load(f)
            if optimizer is not None and meta.get("optimizer_param_groups"):
                for g, sg in zip(optimizer.param_groups, meta["optimizer_param_groups"]):
                    g.update({k: tuple(v) if k == "betas" else v for k, v in sg.items()})
            if scheduler is not None and meta.get("scheduler"):
                scheduler.load_state_dict(meta["scheduler"])
            if meta.get("rng"):
                _set_rng_state(meta["rng"])
            if sampler is not None and meta.get("sampler"):
                sampler.load_state_dict(meta["sampler"])
            out.update(meta)
        return out

    def _load_logical(self, d: Path, model, optimizer):
        """DCP load by logical parameter names into whatever layout this run
        has (TP shards read their chunks, EP ranks their experts, PP stages
        their layers).  Works for model-parallel, replicated and
        reference-written checkpoints alike."""
        from .dcp_state import logical_load_state
        full = getattr(optimizer, "gather_full_state", None)
        if full is not None:
            full()  # full-shape moment views for DCP to load into
        try:
            sd = logical_load_state(model, optimizer)
            if optimizer is not None and not sd.get("optimizer", {}).get("state"):
                sd.pop("optimizer", None)
            dcp.load(sd, checkpoint_id=str(d))
        finally:
            if full is not None:
                optimizer.release_full_state(scatter=True)
        if optimizer is not None and hasattr(optimizer, "step_count"):
            steps = [float(st["step"]) for st in optimizer.state.values() if "step" in st]
            optimizer.step_count = int(max(steps)) if steps else 0

    def _load_plain(self, d, model, optimizer, scheduler):
        st = torch.load(d / "checkpoint.pt", map_location="cpu", weights_only=False)
        model.load_state_dict(st["model"], strict=False)
        if optimizer is not None and "optimizer" in st:
            optimizer.load_state_dict(st["optimizer"])
        if scheduler is not None and "scheduler" in st:
            scheduler.load_state_dict(st["scheduler"])
        extra = dict(st.get("extra", {}))
        extra.setdefault("step", st.get("step", 0))
        return extra

    # ------------------------------------------------------------- helpers
    def latest(self) -> Optional[str]:
        if not self.save_dir.exists():
            return None
        dirs = sorted(self.save_dir.glob("step_*"))
        return str(dirs[-1]) if dirs else None

    def _cleanup(self) -> None:
        dirs = sorted(self.save_dir.glob("step_*"))
        while len(dirs) > self.max_checkpoints:
            shutil.rmtree(dirs.pop(0), ignore_errors=True)
