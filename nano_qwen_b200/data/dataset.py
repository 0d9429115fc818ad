"""Pretraining datasets: memory-mapped packed windows and streaming packing.

``PackedTextDataset`` memory-maps ``*.bin`` token files (uint32 by default) and
serves fixed windows of ``max_seq_len`` tokens (reference:
data/dataset.py:20-93).  Labels are aligned with ``input_ids`` (the model shifts
them), which gives true next-token training; the reference emits pre-shifted
labels that its model shifts again (data/dataset.py:68-69 with
model/transformer.py:140-141), training on token t+2.  Window gathering across
file boundaries is done by the native ``TokenWindowReader`` when the C++ runtime
is built.  With no files the dataset serves seeded uniform-random tokens, the
synthetic path the reference's CLI falls back to (data/dataset.py:46-50).

``DocumentPackingDataset`` packs documents with BOS/EOS separators and also
returns per-token document ids (``doc_ids``) so attention can be restricted to
the document (reference: data/dataset.py:96-146 computed boundaries but did
not emit them).
"""

from __future__ import annotations

import os
from pathlib import Path
from typing import List

import numpy as np
import torch
from torch.utils.data import Dataset, IterableDataset


class PackedTextDataset(Dataset):
    def __init__(self, data_dir: str, max_seq_len: int = 4096, bos_id: int = 151643,
                 eos_id: int = 151645, dtype=np.uint32, vocab_size: int = 32000,
                 synthetic_samples: int = 10000, seed: int = 0):
        self.max_seq_len = max_seq_len
        self.bos_id = bos_id
        self.eos_id = eos_id
        self.vocab_size = vocab_size
        self.seed = seed
        files = sorted(Path(data_dir).glob("*.bin")) if data_dir and os.path.isdir(data_dir) else []
        self.arrays = [np.memmap(f, dtype=dtype, mode="r") for f in files]
        self.bounds = np.cumsum([0] + [a.shape[0] for a in self.arrays])
        self.total_tokens = int(self.bounds[-1])
        self.synthetic = not self.arrays
        if self.synthetic:
            self.num_samples = synthetic_samples
        else:
            self.num_samples = max(self.total_tokens // max_seq_len, 1)
        self._native = None
        if not self.synthetic:
            try:
                from ..runtime.native import TokenWindowReader
                self._native = TokenWindowReader([str(f) for f in files],
                                                 np.dtype(dtype).itemsize, eos_id)
            except Exception:
                self._native = None

    def __len__(self) -> int:
        return self.num_samples

    def _window(self, start: int, n: int) -> np.ndarray:
        if self._native is not None:
            return self._native.read(start, n)
        out = np.empty(n, dtype=np.int64)
        pos, filled = start, 0
        f = int(np.searchsorted(self.bounds, pos, side="right") - 1)
        while filled < n and f < len(self.arrays):
            local = pos - self.bounds[f]
            take = min(n - filled, self.arrays[f].shape[0] - local)
            out[filled:filled + take] = self.arrays[f][local:local + take]
            filled += take
            pos += take
            f += 1
        if filled < n:
            out[filled:] = self.eos_id
        return out

    def __getitem__(self, idx: int) -> dict:
        S = self.max_seq_len
        if self.synthetic:
            g = torch.Generator().manual_seed(self.seed * 1_000_003 + idx)
            tokens = torch.randint(0, self.vocab_size, (S,), generator=g)
        else:
            tokens = torch.from_numpy(self._window(idx * S, S).astype(np.int64))
        return {"input_ids": tokens, "labels": tokens.clone()}


class DocumentPackingDataset(IterableDataset):
    def __init__(self, documents: List[List[int]], max_seq_len: int = 4096,
                 bos_id: int = 151643, eos_id: int = 151645, shuffle: bool = True, seed: int = 42):
        self.documents = documents
        self.max_seq_len = max_seq_len
        self.bos_id = bos_id
        self.eos_id = eos_id
        self.shuffle = shuffle
        self.seed = seed

    def __iter__(self):
        order = np.arange(len(self.documents))
        if self.shuffle:
            np.random.RandomState(self.seed).shuffle(order)
        S = self.max_seq_len
        buf: List[int] = []
        doc: List[int] = []
        next_doc = 0
        for i in order:
            toks = [self.bos_id] + list(self.documents[i]) + [self.eos_id]
            buf.extend(toks)
            doc.extend([next_doc] * len(toks))
            next_doc += 1
            while len(buf) >= S:
                ids = torch.tensor(buf[:S], dtype=torch.long)
                d = torch.tensor(doc[:S], dtype=torch.long)
                d = d - d[0]
                labels = ids.clone()
                # a token's successor in another document is not a target
                labels[1:][d[1:] != d[:-1]] = -100
                buf, doc = buf[S:], doc[S:]
                yield {"input_ids": ids, "labels": labels, "doc_ids": d}
