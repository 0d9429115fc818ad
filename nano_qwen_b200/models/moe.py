"""Qwen3 mixture-of-experts layer.

Same parameters and names as the reference (``router.gate``,
``experts.{e}.ffn.{gate,up,down}_proj``; reference: model/moe.py:23-144).  All
experts' gate|up weights form one contiguous [E*2I, H] fusion group and all
down weights one [E*H, I] group, which the grouped tcgen05 GEMMs consume in a
single launch each.  Routing statistics (counts, probability sums) come out of
the router kernel; the aux loss is the Switch formulation E * sum f_i p_i on the
local batch (reference default) or, when ``global_stats_fn`` is set by the
data-parallel wrapper, with f_i reduced over the global batch.
"""

from __future__ import annotations

from typing import Callable, Optional, Tuple

import torch
import torch.nn as nn

from .. import ops
from ..config import ModelConfig
from .ffn import SwiGLU
from .layers import Linear, fused_linear


class TopKRouter(nn.Module):
    def __init__(self, config: ModelConfig):
        super().__init__()
        self.num_experts = config.num_experts
        self.top_k = config.num_experts_per_tok
        self.norm_topk_prob = config.norm_topk_prob
        self.aux_loss_coef = config.router_aux_loss_coef
        self.gate = Linear(config.hidden_size, config.num_experts, bias=False)
        # < 1 under tensor parallelism: every TP rank computes the same aux loss
        # from the same tokens, so each back-propagates 1/tp of it (the router
        # gradients are summed over TP afterwards).
        self.grad_scale = 1.0

    def forward(self, hidden_states: torch.Tensor):
        """Returns (weights fp32 [N,k], indices int32 [N,k], counts [E], prob_sum [E])."""
        logits = fused_linear(hidden_states, [self.gate], hidden_states.dtype)
        return ops.route(logits, self.top_k, self.norm_topk_prob)


class ExpertFFN(nn.Module):
    def __init__(self, hidden_size: int, intermediate_size: int):
        super().__init__()
        self.ffn = SwiGLU(hidden_size, intermediate_size, bias=False)

    def forward(self, x):
        return self.ffn(x)


class MoELayer(nn.Module):
    def __init__(self, config: ModelConfig):
        super().__init__()
        self.config = config
        self.num_experts = config.num_experts
        self.top_k = config.num_experts_per_tok
        self.drop_tokens = config.moe_drop_tokens
        self.capacity_factor = config.moe_capacity_factor
        self.inter = config.moe_intermediate_size
        self.router = TopKRouter(config)
        self.experts = nn.ModuleList([ExpertFFN(config.hidden_size, config.moe_intermediate_size)
                                      for _ in range(config.num_experts)])
        # Optional hook: (counts [E], num_tokens) -> (global_counts, global_tokens)
        self.global_stats_fn: Optional[Callable] = None
        # Expert parallelism replaces the local expert computation (parallel.expert_parallel)
        self.ep = None

    def fusion_groups(self):
        gu = []
        n = len(self.experts)  # E, or E/ep under expert parallelism
        for e in range(n):
            gu += [f"experts.{e}.ffn.gate_proj.weight", f"experts.{e}.ffn.up_proj.weight"]
        down = [f"experts.{e}.ffn.down_proj.weight" for e in range(n)]
        return [gu, down]

    def expert_weight_refs(self, dtype):
        gu, down = [], []
        for ex in self.experts:
            gu += [ex.ffn.gate_proj.weight, ex.ffn.up_proj.weight]
            down.append(ex.ffn.down_proj.weight)
        return ops.weight_ref(gu, dtype), ops.weight_ref(down, dtype)

    def capacity(self, num_tokens: int) -> Optional[int]:
        if not self.drop_tokens:
            return None
        return int(self.capacity_factor * num_tokens * self.top_k / self.num_experts)

    def forward(self, hidden_states: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        tp = getattr(self, "tp_group", None)
        if tp is not None:
            # experts are sharded along the intermediate dim: all tokens in, partial sums out
            from ..parallel.tensor_parallel import _CopyToTP, gather_seq, scatter_seq, tp_output
            x_in = gather_seq(hidden_states, tp) if self.tp_sp else _CopyToTP.apply(hidden_states, tp)
            out, aux = self._forward_local(x_in)
            out = scatter_seq(out, tp) if self.tp_sp else tp_output_allreduce(out, tp)
            return out, aux
        return self._forward_local(hidden_states)

    def _forward_local(self, hidden_states: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        shape = hidden_states.shape
        x = hidden_states.reshape(-1, shape[-1])
        N = x.shape[0]
        weights, idx, counts, prob_sum = self.router(x)
        gcounts, gtokens = None, None
        if self.global_stats_fn is not None:
            grp = getattr(self, "global_stats_group", None)
            if self.ep is not None and hasattr(self.ep, "covers") and self.ep.covers(grp, x):
                # the fused expert-parallel counts exchange already spans the
                # balancing group: no separate all-reduce in the forward
                gcounts, gtokens = self.ep.global_stats(x, counts, idx.shape[1])
            else:
                gcounts, gtokens = self.global_stats_fn(counts, N)
        aux = ops.aux_loss_from_stats(counts, prob_sum, N, self.top_k, self.num_experts,
                                      gcounts, gtokens)
        if self.router.grad_scale != 1.0:
            from ..parallel.tensor_parallel import scale_grad
            aux = scale_grad(aux, self.router.grad_scale)
        if self.ep is not None:
            out = self.ep(self, x, weights, idx, counts)
        else:
            w_gu, w_d = self.expert_weight_refs(x.dtype)
            out = ops.moe_ffn(x, weights, idx, w_gu, w_d, self.num_experts, self.inter,
                              self.capacity(N))
        return out.view(shape), aux


def tp_output_allreduce(y, group):
    from ..parallel.tensor_parallel import _AllReduce
    return _AllReduce.apply(y, group)


class GlobalBatchLoadBalancer:
    """Accumulates routing statistics over micro-batches (and, via
    ``all_reduce``, over data-parallel ranks) to form the global-batch aux loss
    (reference API: model/moe.py:201-249)."""

    def __init__(self, num_experts: int, top_k: int):
        self.num_experts = num_experts
        self.top_k = top_k
        self.reset()

    def update(self, router_probs: torch.Tensor, expert_indices: torch.Tensor) -> None:
        N = router_probs.shape[0]
        cnt = torch.zeros(self.num_experts, dtype=torch.float32, device=router_probs.device)
        cnt.index_add_(0, expert_indices.reshape(-1).long(),
                       torch.ones(expert_indices.numel(), device=router_probs.device))
        psum = router_probs.float().sum(0)
        self.tokens_per_expert = cnt if self.tokens_per_expert is None else self.tokens_per_expert + cnt
        self.prob_sum_per_expert = psum if self.prob_sum_per_expert is None else self.prob_sum_per_expert + psum
        self.total_tokens += N
        self.num_updates += 1

    def all_reduce(self, group=None) -> None:
        import torch.distributed as dist
        if dist.is_available() and dist.is_initialized() and self.tokens_per_expert is not None:
            t = torch.cat([self.tokens_per_expert, self.prob_sum_per_expert,
                           torch.tensor([float(self.total_tokens)], device=self.tokens_per_expert.device)])
            dist.all_reduce(t, group=group)
            E = self.num_experts
            self.tokens_per_expert, self.prob_sum_per_expert = t[:E], t[E:2 * E]
            self.total_tokens = int(t[-1].item())

    def compute_loss(self) -> torch.Tensor:
        if self.total_tokens == 0:
            return torch.tensor(0.0)
        f = self.tokens_per_expert / (self.total_tokens * self.top_k)
        p = self.prob_sum_per_expert / self.total_tokens
        return self.num_experts * (f * p).sum()

    def reset(self) -> None:
        self.total_tokens = 0
        self.tokens_per_expert = None
        self.prob_sum_per_expert = None
        self.num_updates = 0
