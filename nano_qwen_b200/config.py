"""Model configuration.

The field names, defaults and YAML/JSON surface match the reference's
``ModelConfig`` (reference: model/config.py:12-134) so that the same model
YAML files load unchanged.  Presets mirror model/config.py:141-216.
"""

from __future__ import annotations

import json
from dataclasses import asdict, dataclass, field, fields
from pathlib import Path
from typing import Optional

import yaml


@dataclass
class ModelConfig:
    # core dimensions
    hidden_size: int = 4096
    num_hidden_layers: int = 32
    num_attention_heads: int = 32
    num_key_value_heads: int = 8
    head_dim: Optional[int] = None
    intermediate_size: int = 11008
    vocab_size: int = 151936
    max_position_embeddings: int = 32768
    # normalisation / activation
    rms_norm_eps: float = 1e-6
    hidden_act: str = "silu"
    # attention
    attention_bias: bool = False
    attention_dropout: float = 0.0
    qk_norm: bool = True
    # rotary embedding (rope_scaling={"type": "yarn", "factor": f,
    # "original_max_position_embeddings": n, "mscale": bool})
    rope_theta: float = 1_000_000.0
    rope_scaling: Optional[dict] = None
    # embeddings
    tie_word_embeddings: bool = False
    # mixture of experts
    num_experts: int = 0
    num_experts_per_tok: int = 0
    moe_intermediate_size: int = 0
    decoder_sparse_step: int = 1
    router_aux_loss_coef: float = 0.001
    norm_topk_prob: bool = True
    moe_drop_tokens: bool = False
    moe_capacity_factor: float = 1.25
    # vision tower
    vision_enabled: bool = False
    vision_hidden_size: int = 1024
    vision_num_hidden_layers: int = 24
    vision_num_attention_heads: int = 16
    vision_intermediate_size: int = 4096
    vision_patch_size: int = 14
    vision_image_size: int = 448
    vision_num_channels: int = 3
    vision_deepstack_layers: list = field(default_factory=list)
    vision_merger_spatial_factor: int = 2
    # training
    gradient_checkpointing: bool = False
    initializer_range: float = 0.02
    # special tokens
    bos_token_id: int = 151643
    eos_token_id: int = 151645
    pad_token_id: int = 151643

    def __post_init__(self) -> None:
        if self.head_dim is None:
            self.head_dim = self.hidden_size // self.num_attention_heads

    # ------------------------------------------------------------------ derived
    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0 and self.num_experts_per_tok > 0

    @property
    def num_kv_groups(self) -> int:
        return self.num_attention_heads // self.num_key_value_heads

    @property
    def vision_num_patches(self) -> int:
        side = self.vision_image_size // self.vision_patch_size
        return side * side

    @property
    def q_dim(self) -> int:
        return self.num_attention_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.num_key_value_heads * self.head_dim

    def layer_is_moe(self, layer_idx: int) -> bool:
        """MoE placement rule (reference: model/transformer.py:44-50)."""
        if not self.is_moe or self.decoder_sparse_step <= 0:
            return False
        return layer_idx % self.decoder_sparse_step == 0

    def total_params_estimate(self) -> int:
        """Parameter count estimate (reference: model/config.py:90-111)."""
        h = self.hidden_size
        attn = h * self.q_dim + 2 * h * self.kv_dim + self.q_dim * h
        if self.is_moe:
            ffn = self.num_experts * 3 * h * self.moe_intermediate_size + h * self.num_experts
        else:
            ffn = 3 * h * self.intermediate_size
        per_layer = attn + ffn + 2 * h
        total = self.vocab_size * h + self.num_hidden_layers * per_layer + h
        if not self.tie_word_embeddings:
            total += self.vocab_size * h
        return total

    def active_params_per_token(self, include_embedding: bool = False) -> int:
        """Parameters touched per token (MoE counts top-k experts only)."""
        h = self.hidden_size
        attn = h * self.q_dim + 2 * h * self.kv_dim + self.q_dim * h
        n_moe = sum(1 for i in range(self.num_hidden_layers) if self.layer_is_moe(i))
        n_dense = self.num_hidden_layers - n_moe
        dense_ffn = 3 * h * self.intermediate_size
        moe_ffn = self.num_experts_per_tok * 3 * h * self.moe_intermediate_size + h * self.num_experts
        total = self.num_hidden_layers * attn + n_dense * dense_ffn + n_moe * moe_ffn
        total += self.vocab_size * h  # lm_head GEMM always runs
        if include_embedding:
            total += self.vocab_size * h
        return total

    def train_flops_per_token(self, seq_len: int, causal: bool = True) -> float:
        """6*N_active + attention score/value FLOPs (fwd+bwd) per token."""
        attn_ctx = seq_len / 2 if causal else seq_len
        attn = 12 * self.num_hidden_layers * self.q_dim * attn_ctx
        return 6.0 * self.active_params_per_token() + attn

    # --------------------------------------------------------------------- I/O
    @classmethod
    def from_dict(cls, data: dict) -> "ModelConfig":
        known = {f.name for f in fields(cls)}
        unknown = set(data) - known
        if unknown:
            raise TypeError(f"unknown ModelConfig keys: {sorted(unknown)}")
        return cls(**data)

    @classmethod
    def from_yaml(cls, path: str | Path) -> "ModelConfig":
        with open(path) as f:
            return cls.from_dict(yaml.safe_load(f) or {})

    @classmethod
    def from_json(cls, path: str | Path) -> "ModelConfig":
        with open(path) as f:
            return cls.from_dict(json.load(f))

    def to_dict(self) -> dict:
        return asdict(self)

    def save_yaml(self, path: str | Path) -> None:
        with open(path, "w") as f:
            yaml.safe_dump(self.to_dict(), f, sort_keys=False)

    def save_json(self, path: str | Path) -> None:
        with open(path, "w") as f:
            json.dump(self.to_dict(), f, indent=2)


# ---------------------------------------------------------------------------
# Presets (reference: model/config.py:141-216)
# ---------------------------------------------------------------------------
def debug_config() -> ModelConfig:
    return ModelConfig(hidden_size=256, num_hidden_layers=6, num_attention_heads=8,
                       num_key_value_heads=2, intermediate_size=688, vocab_size=32000,
                       max_position_embeddings=2048, tie_word_embeddings=True,
                       rope_theta=10_000.0)


def debug_moe_config() -> ModelConfig:
    cfg = debug_config()
    cfg.num_experts = 8
    cfg.num_experts_per_tok = 2
    cfg.moe_intermediate_size = 256
    cfg.decoder_sparse_step = 1
    return cfg


def small_config() -> ModelConfig:
    return ModelConfig(hidden_size=2048, num_hidden_layers=28, num_attention_heads=16,
                       num_key_value_heads=8, intermediate_size=5504, vocab_size=151936,
                       max_position_embeddings=32768, tie_word_embeddings=True)


def medium_config() -> ModelConfig:
    return ModelConfig(hidden_size=4096, num_hidden_layers=36, num_attention_heads=32,
                       num_key_value_heads=8, intermediate_size=12288, vocab_size=151936,
                       max_position_embeddings=131072)


def large_moe_config() -> ModelConfig:
    return ModelConfig(hidden_size=4096, num_hidden_layers=94, num_attention_heads=64,
                       num_key_value_heads=4, head_dim=128, intermediate_size=12288,
                       vocab_size=151936, max_position_embeddings=131072, num_experts=128,
                       num_experts_per_tok=8, moe_intermediate_size=1536, decoder_sparse_step=1)


PRESETS = {
    "debug": debug_config,
    "debug_moe": debug_moe_config,
    "small": small_config,
    "medium": medium_config,
    "large": large_moe_config,
}
