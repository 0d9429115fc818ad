"""Autoregressive generation with a preallocated KV cache.

API-compatible with the reference's ``TextGenerator`` (``generate(prompt,
max_new_tokens, temperature, top_k, top_p, repetition_penalty,
enable_thinking, thinking_budget, stop_tokens, stream_callback)`` and
``generate_batch``; reference: eval/generate.py:21-188) with these fixes:

* positions continue from the cache length (the reference restarted RoPE at 0
  for every decode step) and the prompt prefill is causal;
* the cache is a fixed [B, S_max, Hk, D] buffer per layer with device-side
  lengths (no ``torch.cat`` per token), decode attention is the split-K
  sm_100a kernel, and on GPU the whole one-token step (all layers + lm_head) is
  captured once in a CUDA graph and replayed;
* ``sample_batch`` generates many sequences in lockstep (GRPO / online-DPO
  rollouts) and returns per-token log-probs.
"""

from __future__ import annotations

import contextlib

from typing import Callable, List, Optional, Tuple

import torch
import torch.nn.functional as F

from .. import ops
from ..models.kv_cache import StaticKVCache
from ..models.layers import fused_linear


def sample_logits(logits: torch.Tensor, temperature: float, top_k: int, top_p: float,
                  generator: Optional[torch.Generator] = None) -> torch.Tensor:
    """Greedy when temperature == 0, else temperature -> top-k -> top-p sampling
    (the reference's ``_sample``, eval/generate.py:140-170).  logits [B, V]."""
    if temperature == 0:
        return logits.argmax(dim=-1, keepdim=True)
    logits = logits.float() / temperature
    V = logits.shape[-1]
    if top_k and top_k > 0 and top_k < V:
        kth = torch.topk(logits, top_k, dim=-1).values[..., -1:]
        logits = logits.masked_fill(logits < kth, float("-inf"))
    if top_p < 1.0:
        sl, si = torch.sort(logits, descending=True, dim=-1)
        probs = F.softmax(sl, dim=-1)
        remove = probs.cumsum(-1) - probs >= top_p
        sl = sl.masked_fill(remove, float("-inf"))
        logits = torch.full_like(logits, float("-inf")).scatter(1, si, sl)
    probs = F.softmax(logits, dim=-1)
    return torch.multinomial(probs, 1, generator=generator)


class DecodeState:
    """Per-model static caches plus the device-side step inputs."""

    def __init__(self, model, batch: int, max_len: int, device, dtype):
        cfg = model.config
        self.caches = [StaticKVCache(batch, max_len, cfg.num_key_value_heads, cfg.head_dim, dtype,
                                     device) for _ in range(cfg.num_hidden_layers)]
        self.lengths = torch.zeros(batch, dtype=torch.int32, device=device)
        self.ids = torch.zeros(batch, 1, dtype=torch.long, device=device)
        self.max_len = max_len
        self.batch = batch


@torch.no_grad()
def decode_step(model, st: DecodeState) -> torch.Tensor:
    """One token for every sequence: reads st.ids / st.lengths, appends to the
    caches, advances lengths, returns logits [B, V] (fp32)."""
    cfg = model.config
    B = st.batch
    x = ops.embedding(st.ids, model.embed.embed_tokens.weight)  # [B, 1, H] fp32
    pos = st.lengths.long().view(B, 1)
    bidx = torch.arange(B, device=x.device)
    resid, delta = x, None
    eps = cfg.rms_norm_eps
    for layer, cache in zip(model.layers, st.caches):
        resid, h = ops.add_rms_norm(resid, delta, layer.input_layernorm.weight, eps)
        att = layer.attention
        D, Hq, Hk = att.head_dim, att.num_heads, att.num_kv_heads
        qkv = fused_linear(h, [att.q_proj, att.k_proj, att.v_proj], h.dtype)
        qw = att.q_norm.weight if att.qk_norm else None
        kw = att.k_norm.weight if att.qk_norm else None
        q, k, v = ops.rope_qk(qkv, Hq, Hk, D, qw, kw, att.rotary_emb.cos_cached,
                              att.rotary_emb.sin_cached, pos, eps)
        cache.k[bidx, st.lengths.long()] = k[:, 0].to(cache.k.dtype)
        cache.v[bidx, st.lengths.long()] = v[:, 0].to(cache.v.dtype)
        o = ops.decode_attention(q.to(cache.k.dtype).contiguous(), cache.k, cache.v,
                                 st.lengths + 1, st.lengths)
        a = fused_linear(o.reshape(B, 1, Hq * D).to(h.dtype), [att.o_proj], h.dtype)
        resid, h = ops.add_rms_norm(resid, a, layer.post_attention_layernorm.weight, eps)
        if layer._use_moe:
            delta, _ = layer.feed_forward(h)
        else:
            delta = layer.feed_forward(h)
    _, h = ops.add_rms_norm(resid, delta, model.norm.weight, eps)
    logits = ops.linear(h, model.lm_head_ref(h.dtype))[:, 0].float()
    st.lengths.add_(1)
    return logits


@torch.no_grad()
def prefill(model, st: DecodeState, prompt: torch.Tensor) -> torch.Tensor:
    """Prompt [B, P] (same length) -> logits of the last position [B, V]; fills caches."""
    from ..models.kv_cache import KVCache
    B, P = prompt.shape
    caches = [KVCache(capacity=P) for _ in st.caches]
    out = model(prompt, kv_caches=caches, return_logits=True, logits_to_keep=1)
    for c, sc in zip(caches, st.caches):
        kb, vb = c.buffers()
        sc.k[:, :P] = kb[:, :P]
        sc.v[:, :P] = vb[:, :P]
    st.lengths.fill_(P)
    return out["logits"][:, -1].float()


class GraphedDecoder:
    """Captures ``decode_step`` in a CUDA graph (GPU) and replays it."""

    def __init__(self, model, st: DecodeState, use_graph: Optional[bool] = None):
        self.model = model
        self.st = st
        dev = st.ids.device
        self.use_graph = (dev.type == "cuda") if use_graph is None else use_graph
        self.graph = None
        self.out = None

    def __call__(self) -> torch.Tensor:
        if not self.use_graph:
            return decode_step(self.model, self.st)
        if self.graph is None:
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            saved = self.st.lengths.clone()
            with torch.cuda.stream(s):
                for _ in range(2):  # warm up allocations outside the graph
                    decode_step(self.model, self.st)
                    self.st.lengths.copy_(saved)
            torch.cuda.current_stream().wait_stream(s)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                self.out = decode_step(self.model, self.st)
            self.st.lengths.copy_(saved)
        self.graph.replay()
        return self.out


def full_params(model):
    """Context in which a fully sharded model's weights are all gathered and
    kept (the decode step reads the layers' weights directly, and a captured
    CUDA graph needs them at fixed addresses); a no-op otherwise."""
    summon = getattr(getattr(model, "param_store", None), "summon_full_params", None)
    return summon() if summon is not None else contextlib.nullcontext()


class TextGenerator:
    def __init__(self, model, tokenizer, device: torch.device = torch.device("cpu"),
                 max_len: int = 4096, use_graph: Optional[bool] = None):
        self.model = model
        self.tokenizer = tokenizer
        self.device = device
        # never past the RoPE table (positions >= max_position_embeddings have no angles)
        cfg = getattr(model, "config", None)
        mp = getattr(getattr(model, "language_model", model), "config", cfg)
        limit = getattr(mp, "max_position_embeddings", None)
        self.max_len = min(max_len, limit) if limit else max_len
        self.use_graph = use_graph
        self.model.eval()

    def _dtype(self):
        return torch.bfloat16 if self.device.type == "cuda" else torch.float32

    @torch.no_grad()
    def generate(self, prompt: str, max_new_tokens: int = 512, temperature: float = 0.7,
                 top_k: int = 50, top_p: float = 0.9, repetition_penalty: float = 1.0,
                 enable_thinking: bool = False, thinking_budget: Optional[int] = None,
                 stop_tokens: Optional[List[int]] = None,
                 stream_callback: Optional[Callable[[str], None]] = None) -> str:
        with full_params(self.model):
            return self._generate(prompt, max_new_tokens, temperature, top_k, top_p,
                                  repetition_penalty, enable_thinking, thinking_budget,
                                  stop_tokens, stream_callback)

    def _generate(self, prompt, max_new_tokens, temperature, top_k, top_p, repetition_penalty,
                  enable_thinking, thinking_budget, stop_tokens, stream_callback) -> str:
        if enable_thinking:
            prompt = prompt + "<think>\n"
        ids = torch.tensor([self.tokenizer.encode(prompt, allowed_special="all")],
                           dtype=torch.long, device=self.device)
        P = ids.shape[1]
        st = DecodeState(self.model, 1, min(self.max_len, P + max_new_tokens + 8), self.device,
                         self._dtype())
        logits = prefill(self.model, st, ids)
        dec = GraphedDecoder(self.model, st, self.use_graph)
        eos = getattr(self.tokenizer, "eos_id", None)
        stops = set(stop_tokens or [])
        if eos is not None:
            stops.add(eos)
        out: List[int] = []
        think_n, think_done = 0, False
        think_end = self.tokenizer.encode("</think>\n", allowed_special="all") if enable_thinking else []
        for _ in range(max_new_tokens):
            if st.lengths[0].item() >= st.max_len - 1:
                break
            if repetition_penalty != 1.0 and out:
                seen = torch.tensor(sorted(set(out)), device=logits.device)
                vals = logits[0, seen]
                logits[0, seen] = torch.where(vals > 0, vals / repetition_penalty,
                                              vals * repetition_penalty)
            nxt = int(sample_logits(logits, temperature, top_k, top_p)[0, 0])
            if enable_thinking and not think_done:
                think_n += 1
                if thinking_budget and think_n >= thinking_budget:
                    out.extend(think_end)
                    think_done = True
                    for t in think_end:
                        st.ids.fill_(t)
                        logits = dec()
                    continue
            if nxt in stops:
                break
            out.append(nxt)
            if stream_callback is not None:
                stream_callback(self.tokenizer.decode([nxt]))
            if enable_thinking and not think_done and "</think>" in self.tokenizer.decode(out[-10:]):
                think_done = True
            st.ids.fill_(nxt)
            logits = dec()
        return self.tokenizer.decode(out)

    @torch.no_grad()
    def generate_batch(self, prompts: List[str], max_new_tokens: int = 512,
                       temperature: float = 0.7, top_k: int = 50, top_p: float = 0.9) -> List[str]:
        return [self.generate(p, max_new_tokens, temperature, top_k, top_p) for p in prompts]

    @torch.no_grad()
    def sample_batch(self, prompt_ids: torch.Tensor, max_new_tokens: int, temperature: float = 1.0,
                     top_k: int = 0, top_p: float = 1.0, eos_id: Optional[int] = None,
                     check_every: int = 8) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """Lockstep sampling of B sequences sharing a prompt length.

        Returns (tokens [B, T], logprobs [B, T] under the sampling distribution,
        mask [B, T] of tokens before and including the first EOS).
        """
        with full_params(self.model):
            return self._sample_batch(prompt_ids, max_new_tokens, temperature, top_k, top_p,
                                      eos_id, check_every)

    def _sample_batch(self, prompt_ids, max_new_tokens, temperature, top_k, top_p, eos_id,
                      check_every):
        B, P = prompt_ids.shape
        if P >= self.max_len:
            raise ValueError(f"prompt length {P} leaves no room below the {self.max_len}-position limit")
        max_new_tokens = min(max_new_tokens, self.max_len - P)
        st = DecodeState(self.model, B, min(self.max_len, P + max_new_tokens + 8), self.device,
                         self._dtype())
        logits = prefill(self.model, st, prompt_ids.to(self.device))
        dec = GraphedDecoder(self.model, st, self.use_graph)
        toks, lps = [], []
        done = torch.zeros(B, dtype=torch.bool, device=self.device)
        for t in range(max_new_tokens):
            nxt = sample_logits(logits, temperature, top_k, top_p)
            lp = F.log_softmax(logits.float() / max(temperature, 1e-6), -1).gather(1, nxt)
            toks.append(nxt)
            lps.append(lp)
            if eos_id is not None:
                done = done | (nxt[:, 0] == eos_id)
                if (t + 1) % check_every == 0 and bool(done.all()):
                    break
            st.ids.copy_(nxt)
            logits = dec()
        tokens = torch.cat(toks, 1)
        logprobs = torch.cat(lps, 1)
        mask = torch.ones_like(tokens, dtype=torch.bool)
        if eos_id is not None:
            is_eos = (tokens == eos_id).int()
            after = (is_eos.cumsum(1) - is_eos) > 0
            mask = ~after
        return tokens, logprobs, mask
