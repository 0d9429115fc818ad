"""Pipeline parallelism: consecutive transformer blocks on consecutive ranks,
micro-batches scheduled one-forward-one-backward (1F1B).

Stage s of p keeps only its blocks (and the embedding on the first stage, the
final norm and lm_head on the last); activations crossing a stage boundary are
the fp32 residual stream [b, S, H], moved with grouped NCCL send/recv pairs so
that a stage's send of micro-batch i+1 and its receive of the gradient of
micro-batch i never wait on each other.  With tied embeddings the first and
last stages each hold a copy of the shared matrix and exchange their gradients
after the backward pass, so both copies take identical optimizer steps.

The reference only computed a layer split and a split-point spec and never
ran a schedule (reference: distributed/pipeline_parallel.py:28-80); its
``ManualPipelineStage`` is kept below under that name.
"""

from __future__ import annotations

from typing import Dict, List, Optional

import torch
import torch.distributed as dist
import torch.nn as nn

from .. import ops


def split_model_into_stages(model: nn.Module, pp_size: int) -> List[List[int]]:
    """Balanced contiguous layer ranges, earlier stages one longer when the
    count does not divide (reference API: distributed/pipeline_parallel.py:28)."""
    n = len(model.layers)
    per, rem = divmod(n, pp_size)
    out, off = [], 0
    for i in range(pp_size):
        c = per + (1 if i < rem else 0)
        out.append(list(range(off, off + c)))
        off += c
    return out


class PipelineParallel(nn.Module):
    def __init__(self, model: nn.Module, pp_group, pp_ranks: List[int], n_microbatches: int = 4):
        super().__init__()
        from ..models.transformer import Qwen3Model
        if not isinstance(model, Qwen3Model):
            raise TypeError("pipeline parallelism applies to Qwen3Model")
        self.group = pp_group
        self.ranks = list(pp_ranks)
        self.pp = len(self.ranks)
        self.stage = dist.get_rank(pp_group)
        self.first = self.stage == 0
        self.last = self.stage == self.pp - 1
        self.n_micro = max(1, int(n_microbatches))
        self.config = model.config
        cfg = model.config
        self.stage_layers = split_model_into_stages(model, self.pp)
        keep = self.stage_layers[self.stage]
        self.layer_offset = keep[0] if keep else 0
        model.layers = nn.ModuleList([model.layers[i] for i in keep])
        self.tied = bool(cfg.tie_word_embeddings) and self.pp > 1
        if self.tied and self.last and not self.first:
            # own copy of the shared matrix on the last stage (the first stage's
            # values arrive with the initial broadcast below)
            model.lm_head.weight = nn.Parameter(model.embed.embed_tokens.weight.detach().clone())
            # the copy follows the embedding's optimizer rule (no weight
            # decay), or the two stages' copies drift apart
            model.lm_head.weight._no_decay = True
        if not self.first:
            model.embed = None
        if not self.last:
            model.lm_head = None
            model.norm = None
        self.model = model
        self.n_moe_total = sum(1 for i in range(cfg.num_hidden_layers) if cfg.layer_is_moe(i))
        self._pending_sends = []
        if self.tied:
            self._sync_tied(weights=True)
            for r, _ in self._pending_sends:
                r.wait()
            self._pending_sends = []

    # ---------------------------------------------------------------- p2p
    def _peer(self, d: int) -> int:
        return self.ranks[self.stage + d]

    def _p2p(self, send: Optional[torch.Tensor] = None, send_to: Optional[int] = None,
             recv_like: Optional[torch.Tensor] = None, recv_from: Optional[int] = None):
        buf = torch.empty_like(recv_like) if recv_from is not None else None
        ops_ = []
        if send is not None:
            ops_.append(dist.P2POp(dist.isend, send.contiguous(), send_to, self.group))
        if buf is not None:
            ops_.append(dist.P2POp(dist.irecv, buf, recv_from, self.group))
        if not ops_:
            return buf
        if dist.get_backend(self.group) == "nccl":
            reqs = dist.batch_isend_irecv(ops_)
        else:
            reqs = [op.op(op.tensor, op.peer, op.group) for op in ops_]
        if buf is None and dist.get_backend(self.group) == "nccl":
            # send only: the compute stream goes on while NCCL's stream sends;
            # the request (and so the tensor) is kept until the schedule ends
            self._pending_sends.extend((r, send) for r in reqs)
            return buf
        for r in reqs:
            r.wait()
        return buf

    @torch.no_grad()
    def _sync_tied(self, weights: bool = False) -> None:
        """weights=True: last stage takes the first stage's matrix;
        otherwise both stages add the other's gradient."""
        if not (self.first or self.last):
            return
        p = self.model.embed.embed_tokens.weight if self.first else self.model.lm_head.weight
        peer = self.ranks[-1] if self.first else self.ranks[0]
        if weights:
            if self.first:
                self._p2p(send=p.data, send_to=peer)
            else:
                p.data.copy_(self._p2p(recv_like=p.data, recv_from=peer))
            return
        store = getattr(p, "_nq_store", None)
        g = store.grad_of(p) if hasattr(store, "grad_of") else p.grad
        other = self._p2p(send=g, send_to=peer, recv_like=g, recv_from=peer)
        g.add_(other)

    # ------------------------------------------------------------- compute
    def _stage_forward(self, x_in: torch.Tensor, pos, mask=None):
        m = self.model
        gather = getattr(self, "param_gather", None) or getattr(m, "param_gather", None)
        if gather is not None:  # fully sharded: embedding / lm_head / norms gathered
            gather()
        sp = getattr(m, "sp_group", None)
        if self.first:
            # under sequence parallelism a stage holds its TP rank's slice of
            # the sequence, as ``Qwen3Model.hidden`` does
            if sp is not None:
                from .tensor_parallel import split_dim
                x_in = split_dim(x_in, 1, sp)
            resid = m.embed(x_in)
        else:
            resid = x_in
        delta, aux_total = None, None
        for layer in m.layers:
            resid, delta, aux = layer.forward_fused(resid, delta, pos, mask, None, None)
            if aux is not None:
                aux_total = aux if aux_total is None else aux_total + aux
        if self.last:
            _, x = ops.add_rms_norm(resid, delta, m.norm.weight, self.config.rms_norm_eps)
            return x, aux_total
        out = resid if delta is None else resid + delta.to(resid.dtype)
        return out, aux_total

    def pipeline_forward_backward(self, micro_batches: List[Dict[str, torch.Tensor]],
                                  scale: float = 1.0):
        """Runs forward and backward of every micro-batch with the 1F1B order;
        returns (loss, aux) summed over micro-batches, the same on every stage.
        Given several micro-batches, each loss is scaled by 1/m (the mean of
        their means, as the training engine's gradient accumulation); a single
        batch that the pipeline splits itself keeps its token mean (each
        piece weighted by its share of the valid targets)."""
        from ..models.transformer import key_range_mask, shift_targets
        mbs = micro_batches
        split = False
        if len(mbs) == 1 and self.n_micro > 1 and mbs[0]["input_ids"].shape[0] >= self.n_micro:
            split = True
            # split every per-row field (ids, labels, document ids, masks)
            b = mbs[0]
            keys = [k for k, v in b.items() if torch.is_tensor(v) and v.dim() >= 1
                    and v.shape[0] == b["input_ids"].shape[0]]
            parts = {k: b[k].chunk(self.n_micro) for k in keys}
            mbs = [{k: parts[k][j] for k in keys} for j in range(len(parts["input_ids"]))]
        m = len(mbs)
        w = scale / m
        if split:
            counts = [(shift_targets(mb["labels"]) != -100).sum().float() for mb in mbs]
            total = torch.stack(counts).sum().clamp(min=1.0)
            lw = [scale * c / total for c in counts]
        else:
            lw = [w] * m
        coef = self.config.router_aux_loss_coef / max(1, self.n_moe_total)
        dev = mbs[0]["input_ids"].device
        B, S = mbs[0]["input_ids"].shape
        sp = getattr(self.model, "sp_group", None)
        if sp is not None:  # activations between stages are the TP rank's sequence slice
            S //= dist.get_world_size(sp)
        act_like = torch.empty(B, S, self.config.hidden_size, dtype=torch.float32, device=dev)
        saved_in: List[Optional[torch.Tensor]] = [None] * m
        saved_out: List = [None] * m
        loss_sum = torch.zeros((), dtype=torch.float32, device=dev)
        aux_sum = torch.zeros((), dtype=torch.float32, device=dev)

        def fwd(i, a):
            x_in = mbs[i]["input_ids"] if self.first else a.requires_grad_(True)
            # packed documents / padding: the same key ranges as Qwen3Model.forward
            docs = mbs[i].get("document_ids", mbs[i].get("doc_ids"))
            mask = key_range_mask(mbs[i].get("attention_mask"), docs)
            out, aux = self._stage_forward(x_in, None, mask)
            extra = coef * aux * w if aux is not None else None
            if aux is not None:
                aux_sum.add_(aux.detach().float() * w)
            if self.last:
                t = shift_targets(mbs[i]["labels"])
                if sp is not None:
                    from ..models.transformer import _sp_loss
                    loss = _sp_loss(out, self.model.lm_head_ref(out.dtype), t, sp) * lw[i]
                else:
                    loss = ops.linear_cross_entropy(out, self.model.lm_head_ref(out.dtype), t) * lw[i]
                loss_sum.add_(loss.detach().float())
                saved_out[i] = (loss if extra is None else loss + extra, None)
                out = None
            else:
                saved_out[i] = (out, extra)
            saved_in[i] = None if self.first else x_in
            return out

        def bwd(i, g):
            out, extra = saved_out[i]
            if self.last:
                out.backward()
            else:
                ts, gs = [out], [g]
                if extra is not None:
                    ts.append(extra)
                    gs.append(torch.ones_like(extra))
                torch.autograd.backward(ts, gs)
            gin = None if self.first else saved_in[i].grad
            saved_out[i] = None
            saved_in[i] = None
            return gin

        self._pending_sends = []
        prev = None if self.first else self._peer(-1)
        nxt = None if self.last else self._peer(1)
        warm = min(self.pp - self.stage - 1, m)
        for i in range(warm):
            a = self._p2p(recv_like=act_like, recv_from=prev) if prev is not None else None
            out = fwd(i, a)
            self._p2p(send=out, send_to=nxt)
        rest = m - warm
        a = self._p2p(recv_like=act_like, recv_from=prev) if (rest > 0 and prev is not None) else None
        for j in range(rest):
            out = fwd(warm + j, a)
            g = None
            if nxt is not None:
                g = self._p2p(send=out, send_to=nxt, recv_like=act_like, recv_from=nxt)
            gin = bwd(j, g)
            if j == rest - 1:
                if prev is not None:
                    self._p2p(send=gin, send_to=prev)
            elif prev is not None:
                a = self._p2p(send=gin, send_to=prev, recv_like=act_like, recv_from=prev)
        for j in range(rest, m):
            g = self._p2p(recv_like=act_like, recv_from=nxt) if nxt is not None else None
            gin = bwd(j, g)
            if prev is not None:
                self._p2p(send=gin, send_to=prev)
        for r, _ in self._pending_sends:
            r.wait()
        self._pending_sends = []
        if self.tied:
            self._sync_tied()
        # every stage reports the same numbers
        dist.broadcast(loss_sum, src=self.ranks[-1], group=self.group)
        dist.all_reduce(aux_sum, group=self.group)
        return loss_sum, (aux_sum if self.n_moe_total else None)

    def forward(self, *args, **kwargs):
        raise RuntimeError("a pipeline stage runs through pipeline_forward_backward()")

    def duplicated_params(self) -> List[nn.Parameter]:
        """Parameters whose values also live on another stage (counted once in
        the global gradient norm: on the first stage)."""
        if self.tied and self.last and not self.first:
            return [self.model.lm_head.weight]
        return []


def apply_pipeline_parallel(model: nn.Module, pp_group, pp_ranks: List[int],
                            n_microbatches: int = 4) -> PipelineParallel:
    return PipelineParallel(model, pp_group, pp_ranks, n_microbatches)


class ManualPipelineStage(nn.Module):
    """A stage holding a subset of layers (reference API:
    distributed/pipeline_parallel.py:82-130)."""

    def __init__(self, model: nn.Module, layer_indices: List[int], stage_idx: int,
                 is_first: bool = False, is_last: bool = False):
        super().__init__()
        self.stage_idx = stage_idx
        self.is_first, self.is_last = is_first, is_last
        self.layers = nn.ModuleList([model.layers[i] for i in layer_indices])
        if is_first:
            self.embed = model.embed
        if is_last:
            self.norm = model.norm
            self.lm_head = model.lm_head

    def forward(self, hidden_states, position_ids=None, attention_mask=None):
        if self.is_first and hidden_states.dtype == torch.long:
            hidden_states = self.embed(hidden_states)
        aux = []
        for layer in self.layers:
            hidden_states, a = layer(hidden_states, position_ids, attention_mask)
            if a is not None:
                aux.append(a)
        total = sum(aux) if aux else None
        if self.is_last:
            h = self.norm(hidden_states)
            return self.lm_head(h), total
        return hidden_states, total
