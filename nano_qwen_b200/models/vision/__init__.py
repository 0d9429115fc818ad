"""Qwen3-VL vision tower: patch embedding, ViT, DeepStack fusion, spatial
merger and multimodal RoPE."""

from .deepstack import DeepStack
from .merger import VisionMerger
from .mrope import MultimodalRoPE, build_mrope_position_ids, mrope_tables
from .patch_embed import PatchEmbedding
from .vit import ViTAttention, ViTBlock, ViTMLP, VisionTransformer

__all__ = ["DeepStack", "VisionMerger", "MultimodalRoPE", "build_mrope_position_ids",
           "mrope_tables", "PatchEmbedding", "ViTAttention", "ViTBlock", "ViTMLP",
           "VisionTransformer"]
