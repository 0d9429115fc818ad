"""Op layer: every hot op of the framework.

CUDA tensors run the sm_100a kernels of ``nano_qwen_b200._C`` (the extension
must be built; there is no silent fallback).  CPU tensors run the plain
PyTorch statement of the same math (``ops.reference``), which doubles as the
test oracle.
"""

from . import reference
from ._ext import available as native_available
from ._ext import ext
from .attention import KeyRange, attention_core, decode_attention, full_attention, rope_qk
from .embedding import embedding
from .linear import WeightRef, dense, linear, weight_ref
from .loss import linear_cross_entropy, token_logprobs
from .mlp import linear_swiglu, linear_swiglu_supported, swiglu_packed
from .moe import aux_loss_from_stats, moe_ffn, route
from .norm import add_rms_norm, rms_norm
from .vision import gelu, layer_norm, patchify

__all__ = [
    "reference", "native_available", "ext", "KeyRange", "attention_core", "decode_attention",
    "full_attention", "rope_qk", "embedding", "WeightRef", "linear", "weight_ref",
    "linear_cross_entropy", "token_logprobs", "swiglu_packed", "linear_swiglu", "linear_swiglu_supported", "aux_loss_from_stats",
    "moe_ffn", "route", "add_rms_norm", "rms_norm", "gelu", "layer_norm", "patchify",
]
