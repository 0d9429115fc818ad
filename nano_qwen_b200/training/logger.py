"""Rank-0 training logger: stdout, TensorBoard and (optionally) WandB.

Same keys and stdout line as the reference (``train/loss, lr, elapsed_sec, step,
grad_norm, tokens_per_sec, aux_loss`` plus ``dpo/*`` and ``rl/*`` extras;
reference: training/logger.py:12-107), plus ``train/mfu`` when the caller
supplies it.  Throughput passed in here is global tokens per device-timed
second (max over ranks), not the reference's local wall-clock rate.
"""

from __future__ import annotations

import os
import time
from typing import Any, Dict, Optional

from ..parallel.comm import is_main_process


class TrainingLogger:
    def __init__(self, wandb_project: Optional[str] = None, wandb_enabled: bool = False,
                 tensorboard_dir: Optional[str] = None, tensorboard_enabled: bool = True,
                 log_interval: int = 10, jsonl_path: Optional[str] = None):
        self.log_interval = max(1, int(log_interval))
        self._wandb = None
        self._tb = None
        self._jsonl = None
        self._t0 = time.time()
        if not is_main_process():
            return
        if wandb_enabled and wandb_project:
            try:
                import wandb
                wandb.init(project=wandb_project, config={})
                self._wandb = wandb
            except Exception:
                self._wandb = None
        if tensorboard_enabled and tensorboard_dir:
            try:
                from torch.utils.tensorboard import SummaryWriter
                os.makedirs(tensorboard_dir, exist_ok=True)
                self._tb = SummaryWriter(tensorboard_dir)
            except Exception:
                self._tb = None
        if jsonl_path:
            os.makedirs(os.path.dirname(jsonl_path) or ".", exist_ok=True)
            self._jsonl = open(jsonl_path, "a")

    def log(self, metrics: Dict[str, Any], step: int) -> None:
        if not is_main_process():
            return
        if self._wandb is not None:
            self._wandb.log(metrics, step=step)
        if self._tb is not None:
            for k, v in metrics.items():
                if isinstance(v, (int, float)):
                    self._tb.add_scalar(k, v, step)
        if self._jsonl is not None:
            import json
            self._jsonl.write(json.dumps({"step": step, **metrics}) + "\n")
            self._jsonl.flush()

    def log_step(self, step: int, loss: float, lr: float, grad_norm: Optional[float] = None,
                 tokens_per_sec: Optional[float] = None, aux_loss: Optional[float] = None,
                 extra: Optional[Dict[str, Any]] = None, mfu: Optional[float] = None) -> None:
        if step % self.log_interval != 0:
            return
        elapsed = time.time() - self._t0
        m = {"train/loss": loss, "train/lr": lr, "train/elapsed_sec": elapsed, "train/step": step}
        if grad_norm is not None:
            m["train/grad_norm"] = grad_norm
        if tokens_per_sec is not None:
            m["train/tokens_per_sec"] = tokens_per_sec
        if aux_loss is not None:
            m["train/aux_loss"] = aux_loss
        if mfu is not None:
            m["train/mfu"] = mfu
        if extra:
            m.update(extra)
        self.log(m, step)
        if is_main_process():
            parts = [f"step={step}", f"loss={loss:.4f}", f"lr={lr:.2e}"]
            if grad_norm is not None:
                parts.append(f"grad_norm={grad_norm:.4f}")
            if tokens_per_sec is not None:
                parts.append(f"tok/s={tokens_per_sec:.0f}")
            if mfu is not None:
                parts.append(f"mfu={mfu:.3f}")
            if aux_loss is not None:
                parts.append(f"aux_loss={aux_loss:.4f}")
            print(f"[{elapsed:.1f}s] " + " | ".join(parts), flush=True)

    def finish(self) -> None:
        if self._wandb is not None:
            self._wandb.finish()
        if self._tb is not None:
            self._tb.close()
        if self._jsonl is not None:
            self._jsonl.close()
