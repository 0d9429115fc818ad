"""Tokenizer wrapper: tiktoken, sentencepiece, or an offline byte-level codec.

Same interface and special-token table as the reference (``encode(text,
add_bos, add_eos, allowed_special)``, ``decode``, ``bos_id``/``eos_id``,
``vocab_size``, batch variants; reference: data/tokenizer.py:9-111).  The
reference's default tiktoken path downloads ``cl100k_base``; machines without
network (such as the GPU pool) get ``backend="bytes"``: UTF-8 bytes map to ids
0..255 and the special tokens to 256.., which keeps every pipeline runnable
offline.  ``backend="auto"`` picks tiktoken when its encoding is available.
"""

from __future__ import annotations

import os
import re
from typing import List, Optional, Set, Union

SPECIAL_TOKENS = {
    "bos": "<|im_start|>",
    "eos": "<|im_end|>",
    "pad": "<|im_start|>",
    "think_start": "<think>",
    "think_end": "</think>",
    "image_pad": "<|image_pad|>",
    "video_pad": "<|video_pad|>",
    "vision_start": "<|vision_start|>",
    "vision_end": "<|vision_end|>",
}

QWEN_PAT = (r"""(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}{1,3}|"""
            r""" ?[^\s\p{L}\p{N}]+[\r\n]*|\s*[\r\n]+|\s+(?!\S)|\s+""")


class _ByteCodec:
    def __init__(self, specials: List[str]):
        uniq = []
        for s in specials:
            if s not in uniq:
                uniq.append(s)
        self.special_to_id = {s: 256 + i for i, s in enumerate(uniq)}
        self.id_to_special = {v: k for k, v in self.special_to_id.items()}
        self.n_vocab = 256 + len(uniq)
        self._pat = re.compile("(" + "|".join(re.escape(s) for s in
                                             sorted(uniq, key=len, reverse=True)) + ")")

    def encode(self, text: str, allowed_special: Union[str, Set[str]] = ()) -> List[int]:
        if allowed_special == "all":
            allowed = set(self.special_to_id)
        else:
            allowed = set(allowed_special or ())
        out: List[int] = []
        for piece in self._pat.split(text) if allowed else [text]:
            if piece in allowed:
                out.append(self.special_to_id[piece])
            elif piece:
                out.extend(piece.encode("utf-8"))
        return out

    def decode(self, ids: List[int]) -> str:
        buf = bytearray()
        parts: List[str] = []
        for i in ids:
            if i < 256:
                buf.append(i)
            else:
                parts.append(buf.decode("utf-8", errors="replace"))
                buf = bytearray()
                parts.append(self.id_to_special.get(i, ""))
        parts.append(buf.decode("utf-8", errors="replace"))
        return "".join(parts)


class Tokenizer:
    def __init__(self, model_path: Optional[str] = None, backend: str = "auto"):
        self._special = dict(SPECIAL_TOKENS)
        if backend == "auto":
            backend = "tiktoken"
            try:
                self._init_tiktoken(model_path)
            except Exception:
                backend = "bytes"
                self._init_bytes()
        elif backend == "tiktoken":
            try:
                self._init_tiktoken(model_path)
            except Exception:
                backend = "bytes"
                self._init_bytes()
        elif backend == "sentencepiece":
            self._init_sentencepiece(model_path)
        elif backend == "bytes":
            self._init_bytes()
        else:
            raise ValueError(f"Unknown tokenizer backend: {backend}")
        self.backend = backend

    def _init_tiktoken(self, model_path):
        import tiktoken
        if model_path and os.path.exists(model_path):
            ranks = tiktoken.load_tiktoken_bpe(model_path)
            specials = {t: i + len(ranks) for i, t in enumerate(dict.fromkeys(self._special.values()))}
            self._enc = tiktoken.Encoding(name="custom", pat_str=QWEN_PAT, mergeable_ranks=ranks,
                                          special_tokens=specials)
        else:
            self._enc = tiktoken.get_encoding("cl100k_base")
        self._vocab = self._enc.n_vocab

    def _init_sentencepiece(self, model_path):
        import sentencepiece as spm
        if model_path is None:
            raise ValueError("sentencepiece backend requires model_path")
        self._sp = spm.SentencePieceProcessor()
        self._sp.Load(model_path)
        self._vocab = self._sp.GetPieceSize()

    def _init_bytes(self):
        self._enc = _ByteCodec(list(self._special.values()))
        self._vocab = self._enc.n_vocab

    @property
    def vocab_size(self) -> int:
        return self._vocab

    def special_id(self, key: str) -> int:
        return self.encode(self._special[key], allowed_special="all")[0]

    @property
    def bos_id(self) -> int:
        return self.special_id("bos")

    @property
    def eos_id(self) -> int:
        return self.special_id("eos")

    def encode(self, text: str, add_bos: bool = False, add_eos: bool = False,
               allowed_special: Union[str, Set[str]] = set()) -> List[int]:
        if self.backend == "sentencepiece":
            ids = list(self._sp.Encode(text))
        else:
            ids = list(self._enc.encode(text, allowed_special=allowed_special))
        if add_bos:
            ids = [self.bos_id] + ids
        if add_eos:
            ids = ids + [self.eos_id]
        return ids

    def decode(self, ids: List[int]) -> str:
        if self.backend == "sentencepiece":
            return self._sp.Decode(list(ids))
        return self._enc.decode(list(ids))

    def encode_batch(self, texts: List[str], **kw) -> List[List[int]]:
        return [self.encode(t, **kw) for t in texts]

    def decode_batch(self, id_lists: List[List[int]]) -> List[str]:
        return [self.decode(i) for i in id_lists]
