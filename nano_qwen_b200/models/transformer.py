"""Qwen3 decoder: blocks and the full causal language model.

Public API and parameter names match the reference (``Qwen3Model.forward(
input_ids, position_ids, attention_mask, kv_caches, labels) -> {"logits",
"loss", "aux_loss", "hidden_states"}``; reference: model/transformer.py:77-162),
with labels aligned to ``input_ids`` and the model doing the shift.

Execution plan on B200: the residual stream stays fp32 and every residual add
is fused into the following RMSNorm kernel (the model loop carries
``(resid, pending_delta)`` between blocks); the loss is the fused lm_head +
vocab-chunked cross-entropy, so the [T, V] logits are only produced when a
caller asks for them (``return_logits`` / ``logits_to_keep``).
"""

from __future__ import annotations

from typing import List, Optional

import torch
import torch.nn as nn
import torch.utils.checkpoint as ckpt

from .. import ops
from ..config import ModelConfig
from ..utils.tracing import nvtx_range
from .attention import Attention
from .ffn import build_ffn
from .kv_cache import KVCache
from .layers import Linear, RMSNorm
from .moe import MoELayer


class TokenEmbedding(nn.Module):
    """reference: model/embedding.py:9-16 (parameter ``embed_tokens.weight``)."""

    def __init__(self, config: ModelConfig):
        super().__init__()
        self.embed_tokens = nn.Embedding(config.vocab_size, config.hidden_size)
        self.hidden_size = config.hidden_size

    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        return ops.embedding(input_ids, self.embed_tokens.weight)


class _GradReady(torch.autograd.Function):
    """Identity whose backward calls ``hook()`` before passing the gradient on."""

    @staticmethod
    def forward(ctx, x, hook):
        ctx.hook = hook
        return x.view_as(x)

    @staticmethod
    def backward(ctx, g):
        ctx.hook()
        return g, None


class TransformerBlock(nn.Module):
    def __init__(self, config: ModelConfig, layer_idx: int = 0):
        super().__init__()
        self.layer_idx = layer_idx
        self.config = config
        self.input_layernorm = RMSNorm(config.hidden_size, eps=config.rms_norm_eps)
        self.attention = Attention(config, layer_idx)
        self.post_attention_layernorm = RMSNorm(config.hidden_size, eps=config.rms_norm_eps)
        self._use_moe = config.layer_is_moe(layer_idx)
        self.feed_forward = MoELayer(config) if self._use_moe else build_ffn(config)
        # set by data parallelism to overlap gradient reduction with the backward
        self.grad_ready_hook = None
        # set by fully sharded data parallelism: gathers this block's weights
        # before it runs and releases them after (``parallel.fsdp.ParamUnit``)
        self.param_unit = None

    def forward_fused(self, resid: torch.Tensor, delta: Optional[torch.Tensor],
                      position_ids=None, attention_mask=None, kv_cache=None, rope=None):
        """(resid, pending delta) -> (resid, new delta, aux).  resid is fp32."""
        eps = self.config.rms_norm_eps
        unit = self.param_unit
        if unit is not None:
            resid, delta = unit.enter(resid, delta)
        if self.grad_ready_hook is not None and resid.requires_grad:
            # the gradient of the block input is produced after every weight
            # gradient of the block: the hook may start reducing them
            resid = _GradReady.apply(resid, self.grad_ready_hook)
        with nvtx_range(f"layer{self.layer_idx}.attention"):
            resid, x = ops.add_rms_norm(resid, delta, self.input_layernorm.weight, eps)
            a = self.attention(x, position_ids, attention_mask, kv_cache, rope)
        with nvtx_range(f"layer{self.layer_idx}.mlp"):
            resid, x = ops.add_rms_norm(resid, a, self.post_attention_layernorm.weight, eps)
            if self._use_moe:
                f, aux = self.feed_forward(x)
            else:
                f, aux = self.feed_forward(x), None
        if unit is not None:
            resid, f, aux = unit.leave(resid, f, aux)
        return resid, f, aux

    def forward(self, hidden_states, position_ids=None, attention_mask=None, kv_cache=None):
        """Reference-compatible: returns (hidden_states, aux_loss)."""
        resid, f, aux = self.forward_fused(hidden_states.float() if hidden_states.is_cuda
                                           else hidden_states, None, position_ids,
                                           attention_mask, kv_cache)
        return resid + f.to(resid.dtype), aux


def _right_padding(mask) -> bool:
    """True for a 2-D key-padding mask whose real tokens form a prefix of
    every row (or None)."""
    if mask is None:
        return True
    if not (torch.is_tensor(mask) and mask.dim() == 2):
        return False
    m = mask.bool()
    # a prefix: once a row turns false it stays false
    return bool((m[:, 1:] <= m[:, :-1]).all())


def key_range_mask(attention_mask, document_ids=None, cached: bool = False):
    """The attention mask the layers receive: ``document_ids`` or a
    one-run-per-row 2-D padding mask become an ``ops.KeyRange`` (handled by
    the flash-attention kernels); anything else is passed through to the
    general path."""
    if document_ids is not None:
        return ops.KeyRange.from_segments(document_ids)
    if (attention_mask is not None and not cached and torch.is_tensor(attention_mask)
            and attention_mask.dim() == 2
            and attention_mask.dtype in (torch.bool, torch.int32, torch.int64)):
        kr = ops.KeyRange.from_padding_mask(attention_mask)
        if kr is not None:
            return kr
    return attention_mask


class Qwen3Model(nn.Module):
    def __init__(self, config: ModelConfig):
        super().__init__()
        self.config = config
        self.embed = TokenEmbedding(config)
        self.layers = nn.ModuleList([TransformerBlock(config, i)
                                     for i in range(config.num_hidden_layers)])
        self.norm = RMSNorm(config.hidden_size, eps=config.rms_norm_eps)
        self.lm_head = Linear(config.hidden_size, config.vocab_size, bias=False)
        if config.tie_word_embeddings:
            self.lm_head.weight = self.embed.embed_tokens.weight
        self.gradient_checkpointing = config.gradient_checkpointing
        # Set by parallel.tensor_parallel: the residual stream is sequence-sharded.
        self.sp_group = None
        self.tp_group = None
        self.reset_parameters()

    # ------------------------------------------------------------------ init
    @torch.no_grad()
    def reset_parameters(self, generator: Optional[torch.Generator] = None) -> None:
        """Normal(0, initializer_range) for every linear/embedding weight, zeros
        for biases, ones for norms (reference: model/transformer.py:98-105)."""
        std = self.config.initializer_range
        for m in self.modules():
            if isinstance(m, (Linear, nn.Linear)):
                m.weight.normal_(0.0, std, generator=generator)
                if m.bias is not None:
                    m.bias.zero_()
            elif isinstance(m, nn.Embedding):
                m.weight.normal_(0.0, std, generator=generator)

    # --------------------------------------------------------------- forward
    def lm_head_ref(self, dtype):
        return ops.weight_ref([self.lm_head.weight], dtype)

    def compute_dtype(self, device: torch.device) -> torch.dtype:
        return torch.bfloat16 if device.type == "cuda" else self.embed.embed_tokens.weight.dtype

    def hidden(self, input_ids: torch.Tensor, position_ids=None, attention_mask=None,
               kv_caches: Optional[List[KVCache]] = None, inputs_embeds=None, rope=None):
        """Runs embed + blocks + final norm; returns (normed hidden [B,S,H], aux_total, n_moe)."""
        gather = getattr(self, "param_gather", None)
        if gather is not None:  # fully sharded: embedding / lm_head / norms gathered
            gather()
        if self.sp_group is not None:
            # sequence parallel: this rank's slice only (embedding rows are looked
            # up for the local tokens, so their gradient is partial over TP)
            import torch.distributed as dist

            from ..parallel.tensor_parallel import scale_grad, split_dim, split_seq
            if inputs_embeds is None:
                resid = self.embed(split_dim(input_ids, 1, self.sp_group))
            else:
                resid = split_seq(scale_grad(inputs_embeds, 1.0 / dist.get_world_size(self.sp_group)),
                                  self.sp_group)
        else:
            resid = self.embed(input_ids) if inputs_embeds is None else inputs_embeds
        delta = None
        aux_total = None
        n_moe = 0
        use_ckpt = self.gradient_checkpointing and self.training and torch.is_grad_enabled()
        for i, layer in enumerate(self.layers):
            cache = kv_caches[i] if kv_caches is not None else None
            if use_ckpt and cache is None:
                resid, delta, aux = ckpt.checkpoint(layer.forward_fused, resid, delta,
                                                    position_ids, attention_mask, None, rope,
                                                    use_reentrant=False)
            else:
                resid, delta, aux = layer.forward_fused(resid, delta, position_ids,
                                                        attention_mask, cache, rope)
            if aux is not None:
                aux_total = aux if aux_total is None else aux_total + aux
                n_moe += 1
        _, x = ops.add_rms_norm(resid, delta, self.norm.weight, self.config.rms_norm_eps)
        return x, aux_total, n_moe

    def forward(self, input_ids: torch.Tensor, position_ids: Optional[torch.Tensor] = None,
                attention_mask: Optional[torch.Tensor] = None,
                kv_caches: Optional[List[KVCache]] = None, labels: Optional[torch.Tensor] = None,
                return_logits: Optional[bool] = None, logits_to_keep: int = 0,
                inputs_embeds: Optional[torch.Tensor] = None,
                document_ids: Optional[torch.Tensor] = None) -> dict:
        """``document_ids`` [B, S] (optional): a document id per token of
        packed rows; each token then attends only within its document.  A 2-D
        key-padding ``attention_mask`` with one run of real tokens per row
        (left or right padding) runs on the same masked kernels."""
        if (getattr(self, "cp_group", None) is not None and kv_caches is None
                and document_ids is None and _right_padding(attention_mask)):
            # right padding under causal attention: a real token never sees a
            # pad key and the pads' targets are ignored, so plain causal
            # attention is exact for everything the loss reads
            attention_mask = None
        attention_mask = key_range_mask(attention_mask, document_ids, kv_caches is not None)
        if getattr(self, "cp_group", None) is not None and kv_caches is None:
            if attention_mask is not None:
                raise NotImplementedError("context parallelism runs plain causal attention "
                                          "(right-padded rows are accepted; packed documents "
                                          "and left padding are not)")
            return self._forward_cp(input_ids, position_ids, labels, return_logits,
                                    logits_to_keep, inputs_embeds)
        if getattr(self, "tp_fused", False) and kv_caches is None and inputs_embeds is None \
                and position_ids is None and attention_mask is None and input_ids.is_cuda:
            return self._forward_tp_fused(input_ids, labels, return_logits, logits_to_keep)
        x, aux_total, n_moe = self.hidden(input_ids, position_ids, attention_mask, kv_caches,
                                          inputs_embeds)
        dtype = x.dtype
        if return_logits is None:
            return_logits = labels is None
        logits = None
        if return_logits:
            xf = x
            if self.sp_group is not None:
                from ..parallel.tensor_parallel import all_gather_dim
                xf = all_gather_dim(x, 1, self.sp_group)
            xs = xf[:, -logits_to_keep:] if logits_to_keep else xf
            logits = ops.linear(xs, self.lm_head_ref(dtype))
        loss = None
        if labels is not None:
            targets = shift_targets(labels)
            if self.sp_group is None:
                loss = ops.linear_cross_entropy(x, self.lm_head_ref(dtype), targets)
            else:
                loss = _sp_loss(x, self.lm_head_ref(dtype), targets, self.sp_group)
            if n_moe > 0:
                loss = loss + self.config.router_aux_loss_coef * (aux_total / n_moe)
        aux_out = None
        if n_moe > 0:
            aux_out = aux_total
        return {"logits": logits, "loss": loss, "aux_loss": aux_out, "hidden_states": x}

    def _forward_tp_fused(self, input_ids, labels, return_logits, logits_to_keep):
        """Tensor + sequence parallel forward with the all-gathers fused into
        the norms and the reduce-scatters into the row-parallel GEMMs
        (``parallel.tp_fused``); this rank holds tokens [r*R, (r+1)*R) of the
        flattened batch."""
        import torch.distributed as dist

        from ..parallel import tp_fused
        from ..parallel.tensor_parallel import _AllReduce, all_gather_dim
        grp = self.tp_group
        W, r = dist.get_world_size(grp), dist.get_rank(grp)
        B, S = input_ids.shape
        T = B * S
        if T % W:
            raise ValueError("batch tokens must divide by tp_size")
        R = T // W
        comm = getattr(self, "_tp_comm", None)
        if comm is None or comm.R != R:
            comm = self._tp_comm = tp_fused.TPComm(grp, R, self.config.hidden_size, input_ids.device)
        resid = self.embed(input_ids.reshape(-1)[r * R:(r + 1) * R])
        dummy = None
        for i, layer in enumerate(self.layers):
            resid, dummy = tp_fused.block_forward(layer, resid, dummy, comm, i, B, S)
        x = tp_fused.final_norm(resid, dummy, self.norm.weight, comm, self.config.rms_norm_eps)
        dtype = x.dtype
        if return_logits is None:
            return_logits = labels is None
        logits = None
        if return_logits:
            xf = all_gather_dim(x, 0, grp).view(B, S, -1)
            xs = xf[:, -logits_to_keep:] if logits_to_keep else xf
            logits = ops.linear(xs, self.lm_head_ref(dtype))
        loss = None
        if labels is not None:
            t = shift_targets(labels).reshape(-1)[r * R:(r + 1) * R].contiguous()
            n_local = (t != -100).sum().float()
            n_global = n_local.clone()
            dist.all_reduce(n_global, group=grp)
            part = ops.linear_cross_entropy(x, self.lm_head_ref(dtype), t) * \
                (n_local / n_global.clamp(min=1))
            loss = _AllReduce.apply(part, grp)
        return {"logits": logits, "loss": loss, "aux_loss": None, "hidden_states": x}

    def _forward_cp(self, input_ids, position_ids, labels, return_logits, logits_to_keep,
                    inputs_embeds):
        """Context-parallel forward: this rank runs its zigzag share of the
        sequence (``parallel.context_parallel``); the loss is the global mean."""
        import torch.distributed as dist

        from ..parallel.context_parallel import cp_loss, zigzag_indices
        from ..parallel.tensor_parallel import all_gather_dim
        if self.sp_group is not None:
            raise NotImplementedError("context parallelism with sequence parallelism")
        grp = self.cp_group
        ws, r = dist.get_world_size(grp), dist.get_rank(grp)
        src = input_ids if input_ids is not None else inputs_embeds
        B, S = src.shape[0], src.shape[1]
        dev = src.device
        idx = zigzag_indices(S, ws, r, dev)
        pos = (torch.arange(S, device=dev).unsqueeze(0).expand(B, S) if position_ids is None
               else position_ids.expand(B, S))
        x, aux_total, n_moe = self.hidden(
            input_ids[:, idx] if input_ids is not None else None, pos[:, idx], None, None,
            inputs_embeds[:, idx] if inputs_embeds is not None else None)
        dtype = x.dtype
        if return_logits is None:
            return_logits = labels is None
        logits = None
        if return_logits:
            order = torch.cat([zigzag_indices(S, ws, q, dev) for q in range(ws)])
            xg = all_gather_dim(x, 1, grp)
            xf = torch.empty_like(xg)
            xf[:, order] = xg
            xs = xf[:, -logits_to_keep:] if logits_to_keep else xf
            logits = ops.linear(xs, self.lm_head_ref(dtype))
        loss = None
        if labels is not None:
            t = shift_targets(labels)[:, idx].contiguous()
            n_local = (t != -100).sum().float()
            n_global = n_local.clone()
            dist.all_reduce(n_global, group=grp)
            part = ops.linear_cross_entropy(x, self.lm_head_ref(dtype), t) * \
                (n_local / n_global.clamp(min=1))
            loss = cp_loss(part, grp)
            if n_moe > 0:
                loss = loss + self.config.router_aux_loss_coef * (aux_total / n_moe)
        return {"logits": logits, "loss": loss, "aux_loss": aux_total if n_moe > 0 else None,
                "hidden_states": x}

    @torch.no_grad()
    def count_parameters(self) -> dict:
        total = sum(p.numel() for p in self.parameters())
        trainable = sum(p.numel() for p in self.parameters() if p.requires_grad)
        return {"total": total, "trainable": trainable}


def _sp_loss(x, wref, targets, group):
    """Global mean CE when each rank holds a sequence slice: local sum / global
    count, summed over the group (forward all-reduce, identity backward)."""
    import torch.distributed as dist

    from ..parallel.tensor_parallel import _AllReduce, split_dim
    t = split_dim(targets, 1, group)
    n_local = (t != -100).sum().float()
    n_global = n_local.clone()
    dist.all_reduce(n_global, group=group)
    part = ops.linear_cross_entropy(x, wref, t) * (n_local / n_global.clamp(min=1))
    return _AllReduce.apply(part, group)


def shift_targets(labels: torch.Tensor) -> torch.Tensor:
    """targets[:, t] = labels[:, t+1]; the last position is ignored (-100)."""
    pad = torch.full_like(labels[..., :1], -100)
    return torch.cat([labels[..., 1:], pad], dim=-1)
