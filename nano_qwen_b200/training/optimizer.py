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

from typing import List, Optional, Tuple

import torch
import torch.nn as nn

from ..ops._ext import ext
from ..runtime.flat_params import FlatParamStore, no_decay_rule


class FusedAdamW(torch.optim.Optimizer):
    """AdamW on a FlatParamStore.

    ``shard`` = (begin, end) restricts the update to a slice of the flat
    buffers (each data-parallel rank updates its slice and the updated compute
    copy is all-gathered by the caller).  With a proper slice the Adam moments
    are allocated for that slice only (``sharded``): 8 B per parameter divided
    by the data-parallel world instead of 8 B per parameter on every rank.
    Full-shape per-parameter views of the moments (what ``state_dict`` and DCP
    see) then exist only between ``gather_full_state`` and
    ``release_full_state``, which checkpointing calls around a save or load.

    ``pieces`` = [(begin, end), ...]: the flat ranges this rank updates when
    they are not one slice (under expert parallelism the dense shard skips
    the expert span, which is sharded over the ranks holding the same
    experts); the moments are the pieces' elements back to back, and the
    caller performs the update (``step(update=...)``, ``pieces`` then holds
    (begin, end, offset into the moments)).
    """

    pieces: Optional[List[Tuple[int, int, int]]] = None

    def __init__(self, store: FlatParamStore, lr: float = 3e-4, betas=(0.9, 0.95),
                 eps: float = 1e-8, weight_decay: float = 0.1,
                 shard: Optional[Tuple[int, int]] = None,
                 pieces: Optional[List[Tuple[int, int]]] = None):
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
        b, e = self.shard
        self.sharded = (b, e) != (0, store.numel) or pieces is not None
        # flat index of element 0 of exp_avg / exp_avg_sq
        self.state_base = b if self.sharded else 0
        n = e - b if self.sharded else store.numel
        if pieces is not None:
            self.pieces, n = [], 0
            for lo, hi in pieces:
                self.pieces.append((lo, hi, n))
                n += hi - lo
        self.exp_avg = torch.zeros(n, dtype=torch.float32, device=dev)
        self.exp_avg_sq = torch.zeros(n, dtype=torch.float32, device=dev)
        self._full = None
        # completes a full-size buffer across the data-parallel group (set by
        # the training engine; ``gather_full_state`` uses it by default)
        self.state_gather = None
        self.step_count = 0
        self.clip_scale = torch.ones((), dtype=torch.float32, device=dev)
        self.last_grad_norm = torch.zeros((), dtype=torch.float32, device=dev)
        for p in store.params:
            self.state[p] = {"step": torch.zeros((), dtype=torch.float32)}
        if not self.sharded:
            self._bind_views(self.exp_avg, self.exp_avg_sq)

    # ------------------------------------------------------- moment views
    def _ranges(self):
        """(flat begin, flat end, offset into the moments) of this rank's state."""
        if self.pieces is not None:
            return self.pieces
        return [(self.shard[0], self.shard[1], 0)]

    def _bind_views(self, m: torch.Tensor, v: torch.Tensor) -> None:
        for p in self.store.params:
            o = self.store.offset(p)
            self.state[p]["exp_avg"] = m[o:o + p.numel()].view(p.shape)
            self.state[p]["exp_avg_sq"] = v[o:o + p.numel()].view(p.shape)

    @torch.no_grad()
    def gather_full_state(self, gather=None) -> None:
        """Sharded state: build full-size moment buffers (this rank's slice
        filled in, the rest zero), let ``gather(buf)`` complete them across the
        data-parallel group (all-gather), and expose per-parameter views of
        them in ``self.state``.  No-op for unsharded state."""
        if not self.sharded or self._full is not None:
            return
        gather = gather or self.state_gather
        full = []
        for shard in (self.exp_avg, self.exp_avg_sq):
            buf = torch.zeros(self.store.numel, dtype=torch.float32, device=shard.device)
            for lo, hi, off in self._ranges():
                buf[lo:hi].copy_(shard[off:off + hi - lo])
            if gather is not None:
                gather(buf)
            full.append(buf)
        self._full = full
        self._bind_views(*full)

    @torch.no_grad()
    def release_full_state(self, scatter: bool = False) -> None:
        """Drop the full-size buffers of ``gather_full_state``; with
        ``scatter`` first copy this rank's slice of them back into the shard
        (after a load wrote into the views)."""
        if self._full is None:
            return
        if scatter:
            for lo, hi, off in self._ranges():
                self.exp_avg[off:off + hi - lo].copy_(self._full[0][lo:hi])
                self.exp_avg_sq[off:off + hi - lo].copy_(self._full[1][lo:hi])
        for p in self.store.params:
            self.state[p].pop("exp_avg", None)
            self.state[p].pop("exp_avg_sq", None)
        self._full = None

    # ----------------------------------------------------------- clipping
    @torch.no_grad()
    def clip_grad_norm_(self, max_norm: float, norm_sq_reduce=None) -> torch.Tensor:
        """Global L2 norm of the flat gradient (this rank's ranges, optionally
        summed over ranks by ``norm_sq_reduce``); sets the clip factor used by
        step()."""
        sq = None
        for lo, hi, _ in self._ranges():
            g = self.store.grad[lo:hi]
            part = (ext().sum_squares(g) if g.is_cuda
                    else torch.linalg.vector_norm(g).square().reshape(()))
            sq = part if sq is None else sq + part
        if sq is None:
            sq = torch.zeros((), dtype=torch.float32, device=self.store.grad.device)
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
    def step(self, closure=None, update=None):
        """One AdamW step over this rank's range.  ``update(hparams)``, when
        given, performs the update instead of the local kernel (the
        peer-memory data-parallel step fuses it with the all-gather); going
        through ``step`` keeps the LR scheduler's step bookkeeping intact."""
        loss = closure() if closure is not None else None
        st = self.store
        hp = self.advance()
        if update is not None:
            update(hp)
            return loss
        lr_decay, lr_nodecay, beta1, beta2, eps, wd, bc1, bc2 = hp
        for lo, hi, off in self._ranges():
            if hi <= lo:
                continue
            m, v = self.exp_avg[off:], self.exp_avg_sq[off:]
            if st.master.is_cuda:
                comp = st.compute if st.compute is not None else torch.empty(0, device=st.master.device)
                ext().adamw_flat(st.master, st.grad, m, v, comp, self.clip_scale, lo, hi, lo,
                                 st.decay_end, lr_decay, lr_nodecay, beta1, beta2, eps, wd, bc1, bc2)
            else:
                self._step_cpu(lo, hi, m, v, lr_decay, lr_nodecay, beta1, beta2, eps, wd, bc1, bc2)
        return loss

    def _step_cpu(self, b, e, m_all, v_all, lr_d, lr_n, beta1, beta2, eps, wd, bc1, bc2):
        """[b, e) of the store; element b's moments at m_all[0] / v_all[0]."""
        st = self.store
        for lo, hi, lr, w in ((b, min(e, st.decay_end), lr_d, wd),
                              (max(b, st.decay_end), e, lr_n, 0.0)):
            if hi <= lo:
                continue
            p = st.master[lo:hi]
            g = st.grad[lo:hi] * self.clip_scale
            m = m_all[lo - b:hi - b]
            v = v_all[lo - b:hi - b]
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
        """Copy loaded moments into the flat buffers (keeps the views valid);
        sharded state keeps this rank's slice of them."""
        materialized = self.sharded and self._full is None
        if materialized:
            self.gather_full_state()
        try:
            self._load_moments(state_dict)
        finally:
            if materialized:
                self.release_full_state(scatter=True)

    def _load_moments(self, state_dict):
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
                    shard: Optional[Tuple[int, int]] = None,
                    pieces: Optional[List[Tuple[int, int]]] = None) -> torch.optim.Optimizer:
    store = store or getattr(model, "param_store", None)
    if store is not None and getattr(store, "mode", None) == "fsdp":
        from ..parallel.fsdp import FSDPAdamW
        return FSDPAdamW(store, lr=lr, betas=(beta1, beta2), eps=eps, weight_decay=weight_decay)
    if store is not None and fused:
        return FusedAdamW(store, lr=lr, betas=(beta1, beta2), eps=eps,
                          weight_decay=weight_decay, shard=shard, pieces=pieces)
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
