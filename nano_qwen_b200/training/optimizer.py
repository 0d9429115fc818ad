"""AdamW over the flat parameter store, with fused grad-norm clipping.

``build_optimizer`` keeps the reference's signature and decay grouping (no
decay for ndim<=1 and names containing norm/bias/embed; reference:
training/optimizer.py:18-61).  When the model lives in a ``FlatParamStore`` the
step is one sm_100a kernel over the whole store (or over this rank's ZeRO
shard): it reads the fp32 gradient, applies the global clip factor computed on
the device by a fused sum-of-squares kernel (no host sync), updates m, v and
the fp32 master weights, and writes the bf16 compute copy the GEMMs read.
Otherwise it falls back to ``torch.optim.AdamW``.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn as nn

from ..ops._ext import ext
from ..runtime.flat_params import FlatParamStore, no_decay_rule


class FusedAdamW(torch.optim.Optimizer):
    """AdamW on a FlatParamStore.

    ``shard`` = (begin, end) restricts the update to a slice of the flat
    buffers (ZeRO-1 style: each data-parallel rank updates its slice and the
    updated compute copy is all-gathered by the caller).
    """

    def __init__(self, store: FlatParamStore, lr: float = 3e-4, betas=(0.9, 0.95),
                 eps: float = 1e-8, weight_decay: float = 0.1,
                 shard: Optional[Tuple[int, int]] = None):
        self.store = store
        decay = [p for p in store.params if store.offset(p) < store.decay_end]
        nodecay = [p for p in store.params if store.offset(p) >= store.decay_end]
        groups = []
        if decay:
            groups.append({"params": decay, "weight_decay": weight_decay})
        if nodecay:
            groups.append({"params": nodecay, "weight_decay": 0.0})
        super().__init__(groups, dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay))
        dev = store.master.device
        self.shard = shard or (0, store.numel)
        self.exp_avg = torch.zeros(store.numel, dtype=torch.float32, device=dev)
        self.exp_avg_sq = torch.zeros(store.numel, dtype=torch.float32, device=dev)
        self.step_count = 0
        self.clip_scale = torch.ones((), dtype=torch.float32, device=dev)
        self.last_grad_norm = torch.zeros((), dtype=torch.float32, device=dev)
        for p in store.params:
            o = store.offset(p)
            self.state[p] = {
                "step": torch.zeros((), dtype=torch.float32),
                "exp_avg": self.exp_avg[o:o + p.numel()].view(p.shape),
                "exp_avg_sq": self.exp_avg_sq[o:o + p.numel()].view(p.shape),
            }

    # ----------------------------------------------------------- clipping
    @torch.no_grad()
    def clip_grad_norm_(self, max_norm: float, norm_sq_reduce=None) -> torch.Tensor:
        """Global L2 norm of the flat gradient (this shard, optionally summed
        over ranks by ``norm_sq_reduce``); sets the clip factor used by step()."""
        b, e = self.shard
        g = self.store.grad[b:e]
        if g.is_cuda:
            sq = ext().sum_squares(g)
        else:
            sq = (g.double() ** 2).sum().float().reshape(())
        if norm_sq_reduce is not None:
            sq = norm_sq_reduce(sq)
        norm = sq.sqrt()
        self.last_grad_norm = norm
        if max_norm and max_norm > 0:
            self.clip_scale = torch.clamp(max_norm / (norm + 1e-6), max=1.0)
        else:
            self.clip_scale = torch.ones_like(norm)
        return norm

    # --------------------------------------------------------------- step
    def advance(self):
        """Count one step and return this step's hyper-parameters
        (lr_decay, lr_nodecay, beta1, beta2, eps, wd, bc1, bc2)."""
        self.step_count += 1
        t = self.step_count
        g0 = self.param_groups[0]
        beta1, beta2 = g0["betas"]
        wd = g0["weight_decay"] if self.store.decay_end > 0 else 0.0
        for grp in self.param_groups:
            for p in grp["params"]:
                self.state[p]["step"].fill_(t)
        return (g0["lr"], self.param_groups[-1]["lr"], beta1, beta2, g0["eps"], wd,
                1.0 - beta1 ** t, 1.0 - beta2 ** t)

    @torch.no_grad()
    def step(self, closure=None):
        loss = closure() if closure is not None else None
        st = self.store
        b, e = self.shard
        lr_decay, lr_nodecay, beta1, beta2, eps, wd, bc1, bc2 = self.advance()
        if st.master.is_cuda:
            comp = st.compute if st.compute is not None else torch.empty(0, device=st.master.device)
            ext().adamw_flat(st.master, st.grad, self.exp_avg, self.exp_avg_sq, comp,
                             self.clip_scale, b, e, st.decay_end, lr_decay, lr_nodecay, beta1,
                             beta2, eps, wd, bc1, bc2)
        else:
            self._step_cpu(b, e, lr_decay, lr_nodecay, beta1, beta2, eps, wd, bc1, bc2)
        return loss

    def _step_cpu(self, b, e, lr_d, lr_n, beta1, beta2, eps, wd, bc1, bc2):
        st = self.store
        for lo, hi, lr, w in ((b, min(e, st.decay_end), lr_d, wd),
                              (max(b, st.decay_end), e, lr_n, 0.0)):
            if hi <= lo:
                continue
            p = st.master[lo:hi]
            g = st.grad[lo:hi] * self.clip_scale
            m = self.exp_avg[lo:hi]
            v = self.exp_avg_sq[lo:hi]
            p.mul_(1 - lr * w)
            m.mul_(beta1).add_(g, alpha=1 - beta1)
            v.mul_(beta2).addcmul_(g, g, value=1 - beta2)
            denom = (v / bc2).sqrt_().add_(eps)
            p.addcdiv_(m, denom, value=-lr / bc1)
        if st.compute is not None:
            st.compute[b:e].copy_(st.master[b:e])

    def zero_grad(self, set_to_none: bool = False):
        self.store.grad.zero_()

    # ------------------------------------------------------- state dict
    def load_state_dict(self, state_dict):
        """Copy loaded moments into the flat buffers (keeps the views valid)."""
        groups = self.param_groups
        saved_groups = state_dict["param_groups"]
        id_map = {}
        for g, sg in zip(groups, saved_groups):
            for p, pid in zip(g["params"], sg["params"]):
                id_map[pid] = p
            for k, v in sg.items():
                if k != "params":
                    g[k] = v
        max_step = 0
        for pid, s in state_dict["state"].items():
            p = id_map.get(pid)
            if p is None:
                continue
            mine = self.state[p]
            for k in ("exp_avg", "exp_avg_sq"):
                if k in s:
                    mine[k].copy_(s[k].to(mine[k].device, mine[k].dtype).view(mine[k].shape))
            if "step" in s:
                stp = float(s["step"]) if not torch.is_tensor(s["step"]) else float(s["step"].item())
                mine["step"].fill_(stp)
                max_step = max(max_step, int(stp))
        self.step_count = max_step


def build_optimizer(model: nn.Module, lr: float = 3e-4, weight_decay: float = 0.1,
                    beta1: float = 0.9, beta2: float = 0.95, eps: float = 1e-8,
                    fused: bool = True, store: Optional[FlatParamStore] = None,
                    shard: Optional[Tuple[int, int]] = None) -> torch.optim.Optimizer:
    store = store or getattr(model, "param_store", None)
    if store is not None and fused:
        return FusedAdamW(store, lr=lr, betas=(beta1, beta2), eps=eps,
                          weight_decay=weight_decay, shard=shard)
    decay, nodecay = [], []
    for name, p in model.named_parameters():
        if not p.requires_grad:
            continue
        (nodecay if no_decay_rule(name, p) else decay).append(p)
    groups = [{"params": decay, "weight_decay": weight_decay},
              {"params": nodecay, "weight_decay": 0.0}]
    use_fused = fused and torch.cuda.is_available() and all(p.is_cuda for p in decay + nodecay)
    return torch.optim.AdamW(groups, lr=lr, betas=(beta1, beta2), eps=eps, fused=use_fused)


def attach_param_store(model: nn.Module, compute_dtype: Optional[torch.dtype] = None,
                       device: Optional[torch.device] = None,
                       pad_multiple: int = 64, alloc=None) -> FlatParamStore:
    """Re-home a model's trainable parameters into a FlatParamStore."""
    dev = device or next(model.parameters()).device
    if compute_dtype is None:
        compute_dtype = torch.bfloat16 if dev.type == "cuda" else torch.float32
    store = FlatParamStore(model, compute_dtype=compute_dtype, device=dev,
                           pad_multiple=pad_multiple, alloc=alloc)
    model.param_store = store
    return store
