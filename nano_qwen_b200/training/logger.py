"""Training metrics: step statistics fanned out to a list of sinks.

Design.  A trainer hands ``StepLog.record`` the raw step statistics it already
holds, typically 0-d *device* tensors (loss, grad norm, aux loss) that the
training engine returned without synchronising.  Nothing is read back on
steps that are not logged; on a logged step all device scalars are stacked
and copied to the host in one transfer.  The resulting flat metric dict goes
to every sink (stdout line, TensorBoard, WandB, JSON lines), each a small
object with ``write(step, metrics)`` and ``close()``; sinks that cannot start
(a missing package) are dropped with a note instead of failing the run.

Interface kept from the reference (reference: training/logger.py:12-107): the
metric keys ``train/loss, lr, elapsed_sec, step, grad_norm, tokens_per_sec,
aux_loss`` (plus ``dpo/*`` / ``rl/*`` extras passed through ``extra``), the
``[elapsed] step= | loss= | ...`` stdout line, and the ``TrainingLogger``
constructor / ``log`` / ``log_step`` / ``finish`` calls that trainers make.
Throughput is global tokens per device-timed second (max over ranks), and
``train/mfu`` is added when the caller supplies it.
"""

from __future__ import annotations

import json
import os
import sys
import time
from typing import Any, Dict, List, Optional

from ..parallel.comm import is_main_process

# stdout line: key -> (label, format), in print order
_STDOUT_FIELDS = [("train/loss", "loss", "{:.4f}"), ("train/lr", "lr", "{:.2e}"),
                  ("train/grad_norm", "grad_norm", "{:.4f}"),
                  ("train/tokens_per_sec", "tok/s", "{:.0f}"), ("train/mfu", "mfu", "{:.3f}"),
                  ("train/aux_loss", "aux_loss", "{:.4f}")]


class StdoutSink:
    def __init__(self, stream=None):
        self.stream = stream or sys.stdout

    def write(self, step: int, metrics: Dict[str, Any]) -> None:
        parts = [f"step={step}"]
        for key, label, fmt in _STDOUT_FIELDS:
            v = metrics.get(key)
            if isinstance(v, (int, float)):
                parts.append(f"{label}={fmt.format(v)}")
        el = metrics.get("train/elapsed_sec", 0.0)
        print(f"[{el:.1f}s] " + " | ".join(parts), file=self.stream, flush=True)

    def close(self) -> None:
        pass


class JsonlSink:
    def __init__(self, path: str):
        os.makedirs(os.path.dirname(path) or ".", exist_ok=True)
        self.f = open(path, "a")

    def write(self, step: int, metrics: Dict[str, Any]) -> None:
        self.f.write(json.dumps({"step": step, **metrics}) + "\n")
        self.f.flush()

    def close(self) -> None:
        self.f.close()


class TensorBoardSink:
    def __init__(self, log_dir: str):
        from torch.utils.tensorboard import SummaryWriter
        os.makedirs(log_dir, exist_ok=True)
        self.w = SummaryWriter(log_dir)

    def write(self, step: int, metrics: Dict[str, Any]) -> None:
        for k, v in metrics.items():
            if isinstance(v, (int, float)):
                self.w.add_scalar(k, v, step)

    def close(self) -> None:
        self.w.close()


class WandbSink:
    def __init__(self, project: str):
        import wandb
        self.run = wandb.init(project=project, config={})
        self.wandb = wandb

    def write(self, step: int, metrics: Dict[str, Any]) -> None:
        self.wandb.log(metrics, step=step)

    def close(self) -> None:
        self.wandb.finish()


def _try_sink(make, what: str, notes: List[str]):
    try:
        return make()
    except Exception as e:  # optional back-ends: missing package, no network
        notes.append(f"{what} disabled: {e}")
        return None


def host_values(values: Dict[str, Any]) -> Dict[str, Any]:
    """Device scalars -> Python floats in one device-to-host copy; host
    numbers pass through, ``None`` entries are dropped."""
    import torch
    dev_keys = [k for k, v in values.items() if torch.is_tensor(v) and v.numel() == 1]
    out = {k: v for k, v in values.items() if v is not None and k not in dev_keys}
    if dev_keys:
        packed = torch.stack([values[k].detach().reshape(()).float() for k in dev_keys]).cpu()
        out.update(zip(dev_keys, packed.tolist()))
    return out


class TrainingLogger:
    """Rank-0 metric fan-out.  ``sinks`` overrides the sinks that the keyword
    arguments would build (stdout always; TensorBoard, WandB and a JSON-lines
    file when enabled)."""

    def __init__(self, wandb_project: Optional[str] = None, wandb_enabled: bool = False,
                 tensorboard_dir: Optional[str] = None, tensorboard_enabled: bool = True,
                 log_interval: int = 10, jsonl_path: Optional[str] = None,
                 sinks: Optional[list] = None):
        self.log_interval = max(1, int(log_interval))
        self.t_start = time.time()
        self.notes: List[str] = []
        self.sinks: list = []
        if not is_main_process():
            return
        if sinks is not None:
            self.sinks = list(sinks)
            return
        cands = [StdoutSink()]
        if tensorboard_enabled and tensorboard_dir:
            cands.append(_try_sink(lambda: TensorBoardSink(tensorboard_dir), "tensorboard", self.notes))
        if wandb_enabled and wandb_project:
            cands.append(_try_sink(lambda: WandbSink(wandb_project), "wandb", self.notes))
        if jsonl_path:
            cands.append(JsonlSink(jsonl_path))
        self.sinks = [s for s in cands if s is not None]

    def due(self, step: int) -> bool:
        return step % self.log_interval == 0

    def log(self, metrics: Dict[str, Any], step: int) -> None:
        """Write already-formed metrics to every sink except stdout."""
        if not self.sinks:
            return
        m = host_values(metrics)
        for s in self.sinks:
            if not isinstance(s, StdoutSink):
                s.write(step, m)

    def log_step(self, step: int, loss, lr: float, grad_norm=None, tokens_per_sec=None,
                 aux_loss=None, extra: Optional[Dict[str, Any]] = None, mfu=None) -> None:
        """Per-step statistics (floats or 0-d device tensors); only every
        ``log_interval``-th step is read back and written."""
        if not self.due(step) or not self.sinks:
            return
        raw = {"train/loss": loss, "train/lr": lr, "train/grad_norm": grad_norm,
               "train/tokens_per_sec": tokens_per_sec, "train/aux_loss": aux_loss,
               "train/mfu": mfu}
        raw.update(extra or {})
        m = host_values(raw)
        m["train/elapsed_sec"] = time.time() - self.t_start
        m["train/step"] = step
        for s in self.sinks:
            s.write(step, m)

    def finish(self) -> None:
        for s in self.sinks:
            s.close()
        self.sinks = []
