"""Tracing: NVTX ranges and a torch.profiler step hook.

The reference has no tracing beyond wall-clock timestamps in its logger
(reference: training/logger.py:26, :72; training/pretrain.py:154, :194-195).

* ``nvtx_range(name)``: an NVTX range around a region (training step phases,
  each transformer layer's attention and MLP), visible in Nsight Systems or
  any NVTX consumer.  Off unless ``NQ_NVTX=1`` (or ``enable_nvtx(True)``), so
  the hot path pays one boolean test per region.
* ``StepProfiler``: ``torch.profiler`` over a window of training steps
  (``wait`` / ``warmup`` / ``active``), writing a Chrome trace per rank and a
  per-kernel device-time table; driven by the training YAML's ``profiling``
  section (``enabled``, ``wait``, ``warmup``, ``active``, ``dir``).
"""

from __future__ import annotations

import contextlib
import os
from typing import Optional

import torch

_NVTX = os.environ.get("NQ_NVTX", "0") == "1"


def enable_nvtx(on: bool = True) -> None:
    global _NVTX
    _NVTX = bool(on)


def nvtx_enabled() -> bool:
    return _NVTX


@contextlib.contextmanager
def nvtx_range(name: str):
    if not _NVTX or not torch.cuda.is_available():
        yield
        return
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


class StepProfiler:
    """``with prof.step(i): train_step(...)``; profiles steps
    [wait + warmup, wait + warmup + active) and writes
    ``<dir>/trace_rank<r>.json`` plus ``<dir>/kernels_rank<r>.txt``."""

    def __init__(self, out_dir: str, wait: int = 5, warmup: int = 2, active: int = 3,
                 rank: int = 0):
        from torch.profiler import ProfilerActivity, profile, schedule
        self.out_dir = out_dir
        self.rank = rank
        os.makedirs(out_dir, exist_ok=True)
        acts = [ProfilerActivity.CPU]
        if torch.cuda.is_available():
            acts.append(ProfilerActivity.CUDA)
        self.total = wait + warmup + active
        self._steps = 0
        self.prof = profile(activities=acts, schedule=schedule(wait=wait, warmup=warmup, active=active),
                            on_trace_ready=self._ready)
        self.prof.__enter__()
        self.done = False

    def _ready(self, p) -> None:
        p.export_chrome_trace(os.path.join(self.out_dir, f"trace_rank{self.rank}.json"))
        key = "self_cuda_time_total" if torch.cuda.is_available() else "self_cpu_time_total"
        with open(os.path.join(self.out_dir, f"kernels_rank{self.rank}.txt"), "w") as f:
            f.write(p.key_averages().table(sort_by=key, row_limit=40))

    @contextlib.contextmanager
    def step(self, i: int):
        with nvtx_range(f"step {i}"):
            yield
        if not self.done:
            self.prof.step()
            self._steps += 1
            if self._steps >= self.total:
                self.close()

    def close(self) -> None:
        if not self.done:
            self.prof.__exit__(None, None, None)
            self.done = True


def step_profiler_from_config(cfg: Optional[dict], rank: int = 0) -> Optional[StepProfiler]:
    cfg = cfg or {}
    if not cfg.get("enabled", False):
        return None
    return StepProfiler(cfg.get("dir", "profiles_out"), int(cfg.get("wait", 5)), int(cfg.get("warmup", 2)),
                        int(cfg.get("active", 3)), rank)
