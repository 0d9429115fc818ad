"""Image-text samples for the vision-language model.

``ImageProcessor``: bicubic resize, centre crop, CLIP mean/std normalisation
(reference: data/multimodal_dataset.py:37-75).  ``MultimodalDataset`` inserts
``num_merged_tokens`` image-pad tokens (id 151655) at each image position,
builds ``image_token_mask`` and returns the (T, H, W) grid of each image for
MRoPE positions (reference: data/multimodal_dataset.py:78-166).  Labels are
aligned with ``input_ids``; image-pad and padding positions are -100.
"""

from __future__ import annotations

from typing import Dict, List, Optional

import torch
from torch.utils.data import Dataset

try:
    from PIL import Image
    HAS_PIL = True
except Exception:  # pragma: no cover
    HAS_PIL = False

IMAGE_MEAN = [0.48145466, 0.4578275, 0.40821073]
IMAGE_STD = [0.26862954, 0.26130258, 0.27577711]


class ImageProcessor:
    def __init__(self, image_size: int = 448, patch_size: int = 14, mean=None, std=None,
                 merge: int = 2):
        self.image_size = image_size
        self.patch_size = patch_size
        self.merge = merge
        self.mean = torch.tensor(mean or IMAGE_MEAN).view(3, 1, 1)
        self.std = torch.tensor(std or IMAGE_STD).view(3, 1, 1)

    def __call__(self, image) -> torch.Tensor:
        if image is None or not HAS_PIL:
            g = torch.Generator().manual_seed(0)
            return torch.randn(3, self.image_size, self.image_size, generator=g)
        if isinstance(image, str):
            image = Image.open(image)
        image = image.convert("RGB")
        n = self.image_size
        w, h = image.size
        # shorter side -> n, longer side scaled and truncated (the reference's
        # torchvision Resize(n) rule), bicubic; then a centre crop whose offset
        # rounds half to even like the reference's CenterCrop
        size = (n, int(n * h / w)) if w <= h else (int(n * w / h), n)
        if size != (w, h):
            image = image.resize(size, Image.BICUBIC)
        w, h = image.size
        left, top = int(round((w - n) / 2.0)), int(round((h - n) / 2.0))
        image = image.crop((left, top, left + n, top + n))
        import numpy as np
        x = torch.from_numpy(np.asarray(image, dtype="float32") / 255.0).permute(2, 0, 1)
        return (x - self.mean) / self.std

    @property
    def grid(self) -> int:
        return self.image_size // self.patch_size

    @property
    def num_patches(self) -> int:
        return self.grid ** 2

    @property
    def num_merged_tokens(self) -> int:
        return (self.grid // self.merge) ** 2


class MultimodalDataset(Dataset):
    def __init__(self, samples: List[Dict], tokenizer=None,
                 image_processor: Optional[ImageProcessor] = None, max_seq_len: int = 4096,
                 image_token_id: int = 151655):
        self.samples = samples
        self.tokenizer = tokenizer
        self.proc = image_processor or ImageProcessor()
        self.max_seq_len = max_seq_len
        self.image_token_id = image_token_id

    def __len__(self) -> int:
        return len(self.samples)

    def __getitem__(self, idx: int) -> dict:
        s = self.samples[idx]
        text = s.get("text", "")
        if isinstance(text, str):
            ids = self.tokenizer.encode(text) if self.tokenizer is not None else list(range(100))
        else:
            ids = list(text)
        images = s.get("images") or []
        pix = []
        positions = list(s.get("image_positions") or ([0] * len(images)))
        n_img = self.proc.num_merged_tokens
        g = self.proc.grid // self.proc.merge
        out_ids: List[int] = []
        is_img: List[bool] = []
        grids = []
        k = 0
        for i, t in enumerate(ids + [None]):
            while k < len(images) and k < len(positions) and positions[k] == i:
                pix.append(self.proc(images[k]))
                out_ids += [self.image_token_id] * n_img
                is_img += [True] * n_img
                grids.append([1, g, g])
                k += 1
            if t is not None:
                out_ids.append(t)
                is_img.append(False)
        S = self.max_seq_len
        n = min(len(out_ids), S)
        ids_t = torch.zeros(S, dtype=torch.long)
        ids_t[:n] = torch.tensor(out_ids[:n], dtype=torch.long)
        mask = torch.zeros(S, dtype=torch.bool)
        mask[:n] = torch.tensor(is_img[:n], dtype=torch.bool)
        labels = ids_t.clone()
        labels[n:] = -100
        labels[mask] = -100
        out = {"input_ids": ids_t, "labels": labels, "image_token_mask": mask}
        if pix:
            out["pixel_values"] = torch.stack(pix)
            out["image_grid_thw"] = torch.tensor(grids, dtype=torch.long)
        return out
