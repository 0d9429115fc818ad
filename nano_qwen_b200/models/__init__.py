from .attention import Attention
from .ffn import SwiGLU, build_ffn
from .kv_cache import KVCache, StaticKVCache
from .layers import LayerNorm, Linear, RMSNorm
from .moe import ExpertFFN, GlobalBatchLoadBalancer, MoELayer, TopKRouter
from .rope import RotaryEmbedding, apply_rotary_pos_emb, rope_tables
from .transformer import Qwen3Model, TokenEmbedding, TransformerBlock, shift_targets

__all__ = ["Attention", "SwiGLU", "build_ffn", "KVCache", "StaticKVCache", "LayerNorm", "Linear",
           "RMSNorm", "ExpertFFN", "GlobalBatchLoadBalancer", "MoELayer", "TopKRouter",
           "RotaryEmbedding", "apply_rotary_pos_emb", "rope_tables", "Qwen3Model",
           "TokenEmbedding", "TransformerBlock", "shift_targets"]
