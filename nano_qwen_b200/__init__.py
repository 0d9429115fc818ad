"""nano_qwen_b200: a Blackwell-native (sm_100a) Qwen3 dense / MoE / VL training
and inference framework."""

from .config import ModelConfig

__version__ = "0.1.0"
__all__ = ["ModelConfig"]
