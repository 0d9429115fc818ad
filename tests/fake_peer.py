"""A host-side stand-in for the peer-memory runtime, so the host code of the
fused data-parallel step (``parallel/peer_dp.py``) runs on Gloo CPU ranks.

* ``FakeSymmetricAllocator``: every allocation is a file-backed tensor under a
  shared directory, mapped by every rank (the role of symmetric memory); a
  "pointer" is an integer naming (allocator, allocation, rank), resolved by
  the fake kernels.  Allocations happen in the same order on every rank, as
  with the real allocator; ``make_allocator_factory`` gives each allocator a
  directory named by its creation order and its group's ranks, so the groups
  of one layout (the two data-parallel groups of tp2 x dp2, say) and several
  engines in one process never share files.
* ``FakeZeroExt``: the four kernels of the step, restated with tensor
  operations over the mapped buffers: the same flag slots and sequence
  numbers (bounded spin on the peers' flags), the same reads and writes
  (``zero_rs``: mean of every rank's gradient over this rank's shard plus its
  squared norm; ``zero_adamw_ag``: AdamW on the shard, its result cast to the
  compute dtype and stored into every rank's compute copy; ``zero_publish``:
  the barrier before the next forward).
"""

from __future__ import annotations

import os
import time
from typing import Dict, List, Tuple

import torch

_SLOTS = 8


_ALLOCATORS: List["FakeSymmetricAllocator"] = []


def resolve(key: int) -> torch.Tensor:
    return _ALLOCATORS[int(key) >> 20].resolve(key)


def make_allocator_factory(tmp: str):
    """``SymmetricAllocator`` stand-in: ``factory(group)``."""
    count = [0]

    def factory(group=None):
        import torch.distributed as dist
        ranks = (dist.get_process_group_ranks(group) if group is not None
                 else list(range(dist.get_world_size())))
        d = os.path.join(tmp, f"peer{count[0]}_{'-'.join(map(str, ranks))}")
        count[0] += 1
        os.makedirs(d, exist_ok=True)
        return FakeSymmetricAllocator(d, group)
    return factory


class FakeSymmetricAllocator:
    def __init__(self, directory: str, group=None):
        import torch.distributed as dist
        self.dir = directory
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.meta: List[Tuple[int, torch.dtype]] = []
        self.tensors: List[torch.Tensor] = []
        self.id = len(_ALLOCATORS)
        _ALLOCATORS.append(self)

    def path(self, i: int, r: int) -> str:
        return os.path.join(self.dir, f"buf_{i}_{r}")

    def __call__(self, numel: int, dtype: torch.dtype, device) -> torch.Tensor:
        i = len(self.meta)
        self.meta.append((int(numel), dtype))
        t = torch.from_file(self.path(i, self.rank), shared=True, size=int(numel), dtype=dtype)
        t.zero_()
        self.tensors.append(t)
        return t

    def peer_ptrs(self, t: torch.Tensor) -> List[int]:
        i = next(k for k, x in enumerate(self.tensors) if x.data_ptr() == t.data_ptr())
        return [(self.id << 20) | (i << 10) | r for r in range(self.world)]

    def resolve(self, key: int) -> torch.Tensor:
        i, r = (int(key) >> 10) & 1023, int(key) & 1023
        if r == self.rank:
            return self.tensors[i]
        cache: Dict[int, torch.Tensor] = self.__dict__.setdefault("_peers", {})
        if key not in cache:
            numel, dtype = self.meta[i]
            cache[key] = torch.from_file(self.path(i, r), shared=True, size=numel, dtype=dtype)
        return cache[key]


class _Registry:
    resolve = staticmethod(resolve)


class FakeZeroExt:
    """The step's kernels over any fake allocator's buffers (a pointer names
    its allocator)."""

    def __init__(self, alloc=None, timeout_s: float = 30.0):
        self.a = _Registry()
        self.timeout = timeout_s

    def _flags(self, key: int) -> torch.Tensor:
        return self.a.resolve(key).view(torch.int32)

    def _signal(self, p_flags, rank, slot, epoch):
        for key in p_flags:
            self._flags(key)[slot * _SLOTS + rank] = int(epoch)

    def _wait(self, p_flags, rank, slot, epoch):
        mine = self._flags(p_flags[rank])
        t0 = time.time()
        while True:
            if all(int(mine[slot * _SLOTS + s]) >= epoch for s in range(len(p_flags))):
                return
            if time.time() - t0 > self.timeout:
                raise TimeoutError(f"peer flag slot {slot} did not reach {epoch}")
            time.sleep(0.001)

    def zero_rs(self, p_grad, p_comp, p_flags, rank, lo, hi, sq, epoch, ctas, scale):
        self._signal(p_flags, rank, 0, epoch)
        self._wait(p_flags, rank, 0, epoch)
        if hi > lo:
            parts = [self.a.resolve(k)[lo:hi] for k in p_grad]
            mean = torch.stack(parts).sum(0) * (scale / len(parts))
            self.a.resolve(p_grad[rank])[lo:hi] = mean
            sq += mean.double().pow(2).sum().float()

    def zero_clip(self, sq, max_norm, clip, norm):
        n = sq.sqrt().reshape(())
        norm.copy_(n)
        clip.fill_(min(1.0, max_norm / (float(n) + 1e-6)) if max_norm > 0 else 1.0)

    def zero_adamw_ag(self, p_grad, p_comp, p_flags, rank, p, m, v, clip, b, e, sbase, decay_end,
                      lr_d, lr_n, b1, b2, eps, wd, bc1, bc2):
        g = self.a.resolve(p_grad[rank])
        for lo, hi, lr, w in ((b, min(e, decay_end), lr_d, wd), (max(b, decay_end), e, lr_n, 0.0)):
            if hi <= lo:
                continue
            gr = g[lo:hi] * clip
            x = p[lo:hi] * (1 - lr * w)
            mm = m[lo - sbase:hi - sbase]
            vv = v[lo - sbase:hi - sbase]
            mm.mul_(b1).add_(gr, alpha=1 - b1)
            vv.mul_(b2).addcmul_(gr, gr, value=1 - b2)
            p[lo:hi] = x - lr * (mm / bc1) / ((vv / bc2).sqrt() + eps)
        for key in p_comp:
            self.a.resolve(key)[b:e] = p[b:e].to(self.a.resolve(key).dtype)

    def zero_publish(self, p_grad, p_comp, p_flags, rank, epoch):
        self._signal(p_flags, rank, 1, epoch)
        self._wait(p_flags, rank, 1, epoch)

    def error_flag_read(self):
        return 0
