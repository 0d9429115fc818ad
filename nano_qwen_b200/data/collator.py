"""Batch collation (reference: data/collator.py:10-44).

``TextCollator`` stacks equal-length samples and, when ``pin_memory`` is set,
returns page-locked tensors so the trainer's host-to-device copy is an async
DMA.  ``MultimodalCollator`` additionally stacks ``image_token_mask`` and
concatenates ``pixel_values`` across samples.
"""

from __future__ import annotations

from typing import Dict, List

import torch


class TextCollator:
    def __init__(self, pad_id: int = 0, pin_memory: bool = False):
        self.pad_id = pad_id
        self.pin_memory = pin_memory

    def __call__(self, batch: List[Dict]) -> Dict[str, torch.Tensor]:
        out = {k: torch.stack([s[k] for s in batch]) for k in batch[0]
               if isinstance(batch[0][k], torch.Tensor)}
        if self.pin_memory and torch.cuda.is_available():
            out = {k: v.pin_memory() for k, v in out.items()}
        return out


class MultimodalCollator:
    def __init__(self, pad_id: int = 0):
        self.pad_id = pad_id

    def __call__(self, batch: List[Dict]) -> Dict[str, torch.Tensor]:
        out = {
            "input_ids": torch.stack([s["input_ids"] for s in batch]),
            "labels": torch.stack([s["labels"] for s in batch]),
            "image_token_mask": torch.stack([s["image_token_mask"] for s in batch]),
        }
        pv = [s["pixel_values"] for s in batch if "pixel_values" in s]
        if pv:
            out["pixel_values"] = torch.cat(pv, 0)
        return out
