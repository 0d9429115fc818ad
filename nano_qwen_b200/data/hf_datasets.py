"""HuggingFace dataset loaders for every training phase.

Same registries and loader functions as the reference (reference:
data/hf_datasets.py:38-439): pretrain stages 1-3, SFT cold_start / fusion,
GRPO, DPO (UltraFeedback pairing) and multimodal.  Differences: streaming
samples carry labels aligned with ``input_ids`` (the model shifts), DPO padding
is masked out of the labels (-100; the reference left padding id 0 as a label,
data/hf_datasets.py:334-335) and prompt tokens can be masked, and
``load_pretrain_dataset`` is actually used by the pretrain entry point when a
stage's data is requested.  All loaders need network access or a populated HF
cache; trainers fall back to synthetic/dummy data when they fail.
"""

from __future__ import annotations

import re
from typing import Dict, Iterator, List, Optional

import torch
from torch.utils.data import Dataset, IterableDataset

try:
    from datasets import load_dataset
    HAS_DATASETS = True
except Exception:  # pragma: no cover
    HAS_DATASETS = False

PRETRAIN_DATASETS = {
    1: [{"path": "HuggingFaceFW/fineweb", "name": "sample-10BT", "text_col": "text"},
        {"path": "cerebras/SlimPajama-627B", "text_col": "text"}],
    2: [{"path": "open-web-math/open-web-math", "text_col": "text"},
        {"path": "EleutherAI/proof-pile-2", "name": "default", "text_col": "text"}],
    3: [{"path": "emozilla/pg19", "text_col": "text"}],
}
SFT_DATASETS = {
    "cold_start": [
        {"path": "nvidia/OpenMathInstruct-2", "question_col": "problem",
         "answer_col": "generated_solution"},
        {"path": "AI-MO/NuminaMath-CoT", "question_col": "problem", "answer_col": "solution"},
    ],
    "fusion": [
        {"path": "HuggingFaceH4/ultrachat_200k", "messages_col": "messages"},
        {"path": "teknium/OpenHermes-2.5", "messages_col": "conversations"},
    ],
}
GRPO_DATASETS = [
    {"path": "openai/gsm8k", "name": "main", "question_col": "question", "answer_col": "answer"},
    {"path": "lighteval/MATH", "name": "all", "question_col": "problem", "answer_col": "solution"},
]
DPO_DATASETS = [{"path": "openbmb/UltraFeedback", "name": "default"}]
MULTIMODAL_DATASETS = [{"path": "liuhaotian/LLaVA-Instruct-150K"}]


def _require():
    if not HAS_DATASETS:
        raise ImportError("the `datasets` package is required for HF loaders")


class StreamingTextDataset(IterableDataset):
    """Round-robin over HF streams, tokenise and pack into ``max_seq_len`` windows."""

    def __init__(self, hf_configs: List[dict], tokenizer, max_seq_len: int = 4096, seed: int = 42):
        self.hf_configs = hf_configs
        self.tokenizer = tokenizer
        self.max_seq_len = max_seq_len
        self.seed = seed

    def __iter__(self) -> Iterator[dict]:
        _require()
        streams = []
        for cfg in self.hf_configs:
            kw = {"streaming": True, "split": "train"}
            if "name" in cfg:
                kw["name"] = cfg["name"]
            streams.append((iter(load_dataset(cfg["path"], **kw)), cfg.get("text_col", "text")))
        buf: List[int] = []
        i = 0
        while streams:
            it, col = streams[i % len(streams)]
            try:
                row = next(it)
            except StopIteration:
                streams.pop(i % len(streams))
                continue
            i += 1
            text = row.get(col) or ""
            if not text:
                continue
            buf.extend(self.tokenizer.encode(text) + [self.tokenizer.eos_id])
            while len(buf) >= self.max_seq_len:
                ids = torch.tensor(buf[: self.max_seq_len], dtype=torch.long)
                buf = buf[self.max_seq_len:]
                yield {"input_ids": ids, "labels": ids.clone()}


def load_pretrain_dataset(stage: int, tokenizer, max_seq_len: int = 4096) -> IterableDataset:
    _require()
    return StreamingTextDataset(PRETRAIN_DATASETS.get(stage, PRETRAIN_DATASETS[1]), tokenizer,
                                max_seq_len)


def _extract_answer_number(text: str) -> str:
    m = re.findall(r"####\s*(.+)", text)
    if m:
        return m[-1].strip()
    nums = re.findall(r"-?\d+\.?\d*", text)
    return nums[-1] if nums else text.strip()


def _qa_samples(ds, qcol, acol, max_samples=None, with_reasoning=True) -> List[Dict]:
    out = []
    for i, row in enumerate(ds):
        if max_samples and i >= max_samples:
            break
        q, a = row.get(qcol, ""), row.get(acol, "")
        if not q or not a:
            continue
        turn = {"user": q, "assistant": _extract_answer_number(a) if "####" in a else a}
        if with_reasoning:
            turn["reasoning"] = a
        out.append({"conversations": [turn]})
    return out


def _message_samples(ds, col, max_samples=None) -> List[Dict]:
    out = []
    for i, row in enumerate(ds):
        if max_samples and i >= max_samples:
            break
        msgs = row.get(col, []) or []
        convs = []
        for j in range(0, len(msgs) - 1, 2):
            u, a = msgs[j], msgs[j + 1]
            uc = u.get("content", u.get("value", "")) if isinstance(u, dict) else str(u)
            ac = a.get("content", a.get("value", "")) if isinstance(a, dict) else str(a)
            if uc and ac:
                convs.append({"user": uc, "assistant": ac})
        if convs:
            out.append({"conversations": convs})
    return out


def load_sft_dataset(variant: str, tokenizer, max_seq_len: int = 8192,
                     max_samples: Optional[int] = None, thinking_enabled: bool = True) -> Dataset:
    _require()
    from ..training.sft import SFTDataset
    samples: List[Dict] = []
    for cfg in SFT_DATASETS.get(variant, SFT_DATASETS["cold_start"]):
        kw = {"split": "train"}
        if "name" in cfg:
            kw["name"] = cfg["name"]
        ds = load_dataset(cfg["path"], **kw)
        if "question_col" in cfg:
            samples += _qa_samples(ds, cfg["question_col"], cfg["answer_col"], max_samples,
                                   with_reasoning=(variant == "cold_start"))
        else:
            samples += _message_samples(ds, cfg["messages_col"], max_samples)
    if max_samples:
        samples = samples[:max_samples]
    return SFTDataset(samples, tokenizer, max_seq_len, thinking_enabled=thinking_enabled)


def load_grpo_dataset(max_samples: Optional[int] = None) -> List[Dict]:
    _require()
    out: List[Dict] = []
    for cfg in GRPO_DATASETS:
        kw = {"split": "train"}
        if "name" in cfg:
            kw["name"] = cfg["name"]
        ds = load_dataset(cfg["path"], **kw)
        for i, row in enumerate(ds):
            if max_samples and i >= max_samples:
                break
            q, a = row.get(cfg["question_col"], ""), row.get(cfg["answer_col"], "")
            if q and a:
                out.append({"prompt": q, "answer": _extract_answer_number(a)})
    return out[:max_samples] if max_samples else out


class DPODataset(Dataset):
    """Chosen/rejected pairs; labels are ids with padding (and optionally the
    shared prompt) set to -100."""

    def __init__(self, pairs: List[Dict], tokenizer, max_seq_len: int = 2048,
                 pad_id: int = 0, mask_prompt: bool = False):
        self.pairs = pairs
        self.tokenizer = tokenizer
        self.max_seq_len = max_seq_len
        self.pad_id = pad_id
        self.mask_prompt = mask_prompt

    def __len__(self) -> int:
        return len(self.pairs)

    def _tok(self, text: str, prompt_len: int = 0):
        ids = self.tokenizer.encode(text, allowed_special="all")[: self.max_seq_len]
        n = len(ids)
        ids = ids + [self.pad_id] * (self.max_seq_len - n)
        t = torch.tensor(ids, dtype=torch.long)
        lab = t.clone()
        lab[n:] = -100
        if self.mask_prompt and prompt_len:
            lab[:min(prompt_len, n)] = -100
        return t, lab

    def __getitem__(self, idx: int) -> dict:
        p = self.pairs[idx]
        plen = len(self.tokenizer.encode(p["prompt"], allowed_special="all")) if "prompt" in p else 0
        c, cl = self._tok(p["chosen"], plen)
        r, rl = self._tok(p["rejected"], plen)
        return {"chosen_ids": c, "rejected_ids": r, "chosen_labels": cl, "rejected_labels": rl}


def _ultrafeedback_pairs(ds) -> List[Dict]:
    pairs = []
    for row in ds:
        scored = []
        for c in row.get("completions", []) or []:
            r = c.get("overall_score", c.get("fine-grained_score", 0))
            try:
                r = float(r)
            except (TypeError, ValueError):
                r = 0.0
            if c.get("response"):
                scored.append((r, c["response"]))
        if len(scored) < 2:
            continue
        scored.sort(key=lambda x: x[0], reverse=True)
        ins = row.get("instruction", "")
        prompt = f"User: {ins}\nAssistant: "
        pairs.append({"prompt": prompt, "chosen": prompt + scored[0][1],
                      "rejected": prompt + scored[-1][1]})
    return pairs


def load_dpo_dataset(tokenizer, max_seq_len: int = 2048, max_samples: Optional[int] = None):
    _require()
    pairs: List[Dict] = []
    for cfg in DPO_DATASETS:
        kw = {"split": "train"}
        if "name" in cfg:
            kw["name"] = cfg["name"]
        ds = load_dataset(cfg["path"], **kw)
        if "UltraFeedback" in cfg["path"]:
            pairs += _ultrafeedback_pairs(ds)
        else:
            pairs += [{"chosen": r["chosen"], "rejected": r["rejected"]} for r in ds
                      if r.get("chosen") and r.get("rejected")]
    if max_samples:
        pairs = pairs[:max_samples]
    return DPODataset(pairs, tokenizer, max_seq_len)


def load_multimodal_dataset(tokenizer, image_processor=None, max_seq_len: int = 4096,
                            max_samples: Optional[int] = None):
    _require()
    from .multimodal_dataset import ImageProcessor, MultimodalDataset
    ds = load_dataset(MULTIMODAL_DATASETS[0]["path"], split="train")
    samples = []
    for i, row in enumerate(ds):
        if max_samples and i >= max_samples:
            break
        convs = row.get("conversations", []) or []
        text = " ".join(c.get("value", "") for c in convs if c.get("from") in ("human", "user"))
        img = row.get("image")
        samples.append({"text": text, "images": [img] if img is not None else [],
                        "image_positions": [0] if img is not None else []})
    return MultimodalDataset(samples, tokenizer, image_processor or ImageProcessor(), max_seq_len)
