"""Process-group bootstrap and collective helpers.

Same helper surface as the reference (reference: distributed/comm.py:12-116):
``init_distributed``, rank/world queries, ``barrier``, ``all_reduce_mean/sum``,
``all_gather_tensors``, ``AsyncAllReduce``, ``all_to_all``.  Differences:

* backend is NCCL when CUDA is available and Gloo otherwise, so the same code
  runs the multi-rank CPU tests;
* the process-group timeout defaults to 10 minutes (``NQ_PG_TIMEOUT_S``), not
  30, so ranks waiting on a dead peer fail quickly;
* rendezvous defaults to 127.0.0.1 when MASTER_ADDR is unset.
"""

from __future__ import annotations

import datetime
import os
from typing import List, Optional

import torch
import torch.distributed as dist


def init_distributed(backend: Optional[str] = None, timeout_minutes: Optional[float] = None):
    """Initialise the default process group from the torchrun environment.

    Returns (rank, world_size).  A no-op when WORLD_SIZE is 1 or already set up.
    """
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if world > 1:
        use_cuda = torch.cuda.is_available()
        backend = backend or ("nccl" if use_cuda else "gloo")
        if use_cuda:
            torch.cuda.set_device(local)
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29500")
        if timeout_minutes is None:
            secs = float(os.environ.get("NQ_PG_TIMEOUT_S", 600))
        else:
            secs = timeout_minutes * 60.0
        kwargs = {}
        if backend == "nccl":
            kwargs["device_id"] = torch.device("cuda", local)
        dist.init_process_group(backend=backend, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=secs), **kwargs)
    return rank, world


def is_dist() -> bool:
    return dist.is_available() and dist.is_initialized()


def get_rank(group=None) -> int:
    return dist.get_rank(group) if is_dist() else 0


def get_world_size(group=None) -> int:
    return dist.get_world_size(group) if is_dist() else 1


def get_local_rank() -> int:
    return int(os.environ.get("LOCAL_RANK", 0))


def is_main_process() -> bool:
    return get_rank() == 0


def barrier(group=None) -> None:
    if is_dist():
        if dist.get_backend(group) == "nccl":
            dist.barrier(group=group, device_ids=[torch.cuda.current_device()])
        else:
            dist.barrier(group=group)


def all_reduce_sum(t: torch.Tensor, group=None) -> torch.Tensor:
    if is_dist() and get_world_size(group) > 1:
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    return t


def all_reduce_mean(t: torch.Tensor, group=None) -> torch.Tensor:
    if is_dist() and get_world_size(group) > 1:
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
        t /= get_world_size(group)
    return t


def all_reduce_max(t: torch.Tensor, group=None) -> torch.Tensor:
    if is_dist() and get_world_size(group) > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return t


def all_gather_tensors(t: torch.Tensor, group=None) -> List[torch.Tensor]:
    if not is_dist() or get_world_size(group) == 1:
        return [t]
    out = [torch.empty_like(t) for _ in range(get_world_size(group))]
    dist.all_gather(out, t, group=group)
    return out


class AsyncAllReduce:
    """Non-blocking all-reduce whose completion is awaited later."""

    def __init__(self):
        self._work = None
        self._t = None

    def start(self, t: torch.Tensor, op=None, group=None) -> None:
        self._t = t
        if is_dist() and get_world_size(group) > 1:
            self._work = dist.all_reduce(t, op=op or dist.ReduceOp.SUM, group=group, async_op=True)

    def wait(self) -> torch.Tensor:
        if self._work is not None:
            self._work.wait()
            self._work = None
        return self._t


def all_to_all(outputs: List[torch.Tensor], inputs: List[torch.Tensor], group=None) -> None:
    if not is_dist() or get_world_size(group) == 1:
        for o, i in zip(outputs, inputs):
            o.copy_(i)
        return
    dist.all_to_all(outputs, inputs, group=group)


def max_over_ranks(value: float, device=None) -> float:
    """Max of a host float over all ranks (used for device-timed step times)."""
    if not is_dist():
        return value
    dev = device or (torch.device("cuda", torch.cuda.current_device())
                     if torch.cuda.is_available() and dist.get_backend() == "nccl" else "cpu")
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------------------
# Flat-buffer collectives used by data parallelism.  NCCL runs them natively;
# Gloo (the CPU test backend) has no AVG op, no reduce-scatter and no
# all-gather into one tensor, so they are emulated there.
def _nccl(group) -> bool:
    return dist.get_backend(group) == "nccl"


def all_reduce_avg_(t: torch.Tensor, group=None) -> torch.Tensor:
    if _nccl(group):
        dist.all_reduce(t, op=dist.ReduceOp.AVG, group=group)
    else:
        dist.all_reduce(t, group=group)
        t.div_(dist.get_world_size(group))
    return t


def reduce_scatter_avg_(out: torch.Tensor, inp: torch.Tensor, group=None) -> torch.Tensor:
    """out = mean over ranks of inp's chunk for this rank (out may alias inp)."""
    if _nccl(group):
        dist.reduce_scatter_tensor(out, inp, op=dist.ReduceOp.AVG, group=group)
        return out
    ws, r = dist.get_world_size(group), dist.get_rank(group)
    tmp = inp.clone()
    dist.all_reduce(tmp, group=group)
    n = out.numel()
    out.copy_(tmp[r * n:(r + 1) * n].view_as(out) / ws)
    return out


def all_gather_flat_(out: torch.Tensor, inp: torch.Tensor, group=None) -> torch.Tensor:
    """out = concatenation over ranks of inp."""
    if _nccl(group):
        dist.all_gather_into_tensor(out, inp, group=group)
        return out
    parts = [torch.empty_like(inp) for _ in range(dist.get_world_size(group))]
    dist.all_gather(parts, inp.contiguous(), group=group)
    out.copy_(torch.cat(parts).view_as(out))
    return out
