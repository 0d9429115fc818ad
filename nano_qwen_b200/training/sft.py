"""Supervised fine-tuning: long-CoT cold start and thinking-mode fusion.

Same chat template, ``format_conversation``, ``SFTDataset``,
``ThinkingModeFusion`` and ``run_sft`` surface as the reference
(training/sft.py:39-404).  Differences:

* assistant-only loss masks are exact at the token level: the conversation is
  tokenised segment by segment, so labels cover precisely the assistant tokens
  (the reference approximated token positions from a character ratio,
  training/sft.py:137-146);
* labels are aligned with ``input_ids`` (the model shifts) and padding is -100;
* the ``sft.think_token`` / ``sft.no_think_token`` / ``sft.mask_input`` YAML
  keys are honoured (the reference ignored them);
* the step loop is the fused ``TrainEngine``.
"""

from __future__ import annotations

import random
from typing import Dict, List, Optional

import torch
import yaml
from torch.utils.data import DataLoader, Dataset

from ..config import ModelConfig
from ..data.collator import TextCollator
from ..data.sampler import DistributedSampler
from ..data.tokenizer import Tokenizer
from ..models.transformer import Qwen3Model
from ..parallel.comm import init_distributed, is_main_process
from .checkpoint import CheckpointManager, resolve_resume
from .engine import TrainEngine
from .logger import TrainingLogger
from .pretrain import pick_device

CHAT_TEMPLATE = ("<|im_start|>system\n{system}<|im_end|>\n"
                 "<|im_start|>user\n{user}<|im_end|>\n"
                 "<|im_start|>assistant\n{assistant}<|im_end|>")
THINK_TEMPLATE = "{open}\n{reasoning}\n{close}\n{answer}"
NO_THINK_TEMPLATE = "{open}\n{close}\n{answer}"


def assistant_text(assistant: str, reasoning: Optional[str], enable_thinking: bool,
                   think_open: str = "<think>", think_close: str = "</think>") -> str:
    if enable_thinking and reasoning:
        return THINK_TEMPLATE.format(open=think_open, close=think_close, reasoning=reasoning,
                                     answer=assistant)
    if enable_thinking:
        return NO_THINK_TEMPLATE.format(open=think_open, close=think_close, answer=assistant)
    return assistant


def format_conversation(system: str, user: str, assistant: str, reasoning: Optional[str] = None,
                        enable_thinking: bool = True) -> str:
    """reference: training/sft.py:49-68."""
    return CHAT_TEMPLATE.format(system=system, user=user,
                                assistant=assistant_text(assistant, reasoning, enable_thinking))


class SFTDataset(Dataset):
    def __init__(self, samples: List[Dict], tokenizer, max_seq_len: int = 8192,
                 mask_input: bool = True, thinking_enabled: bool = True,
                 system_prompt: str = "You are a helpful assistant.", think_open: str = "<think>",
                 think_close: str = "</think>", pad_id: int = 0):
        self.samples = samples
        self.tokenizer = tokenizer
        self.max_seq_len = max_seq_len
        self.mask_input = mask_input
        self.thinking_enabled = thinking_enabled
        self.system_prompt = system_prompt
        self.think_open = think_open
        self.think_close = think_close
        self.pad_id = pad_id

    def __len__(self) -> int:
        return len(self.samples)

    def _enc(self, text: str) -> List[int]:
        return self.tokenizer.encode(text, allowed_special="all")

    def segments(self, sample: Dict):
        """[(token_ids, is_assistant)] for one conversation."""
        system = sample.get("system", self.system_prompt)
        segs = []
        for turn in sample.get("conversations", []):
            prefix = (f"<|im_start|>system\n{system}<|im_end|>\n"
                      f"<|im_start|>user\n{turn['user']}<|im_end|>\n<|im_start|>assistant\n")
            body = assistant_text(turn["assistant"], turn.get("reasoning"), self.thinking_enabled,
                                  self.think_open, self.think_close) + "<|im_end|>"
            segs.append((self._enc(prefix), False))
            segs.append((self._enc(body), True))
            segs.append((self._enc("\n"), False))
        return segs

    def __getitem__(self, idx: int) -> dict:
        ids: List[int] = []
        lab: List[int] = []
        for toks, is_asst in self.segments(self.samples[idx]):
            ids.extend(toks)
            lab.extend(toks if (is_asst or not self.mask_input) else [-100] * len(toks))
        S = self.max_seq_len
        ids, lab = ids[:S], lab[:S]
        n = len(ids)
        ids = ids + [self.pad_id] * (S - n)
        lab = lab + [-100] * (S - n)
        return {"input_ids": torch.tensor(ids, dtype=torch.long),
                "labels": torch.tensor(lab, dtype=torch.long)}


class SFTTrainer:
    def __init__(self, model, training_config: dict, device: torch.device, parallel=None):
        """``parallel``: the ``ParallelismManager`` the model went through
        (tensor / pipeline / expert / context parallelism from the training
        YAML's ``distributed`` section, as in pretraining)."""
        self.cfg = training_config
        self.device = device
        self.engine = TrainEngine(model, training_config, device, parallel=parallel)
        self.model = self.engine.model
        self.optimizer = self.engine.optimizer
        self.scheduler = self.engine.scheduler
        ck = training_config.get("checkpoint", {}) or {}
        self.ckpt_mgr = CheckpointManager(save_dir=ck.get("save_dir", "checkpoints/sft"),
                                          save_interval=ck.get("save_interval", 500),
                                          async_save=ck.get("async_save", True))
        lg = training_config.get("logging", {}) or {}
        self.logger = TrainingLogger(wandb_project=lg.get("wandb_project"),
                                     wandb_enabled=lg.get("wandb_enabled", False),
                                     tensorboard_dir=lg.get("tensorboard_dir"),
                                     tensorboard_enabled=lg.get("tensorboard_enabled", True),
                                     log_interval=lg.get("log_interval", 10))
        self.grad_accum_steps = (training_config.get("batch", {}) or {}).get(
            "gradient_accumulation_steps", 1)

    def train(self, dataloader, total_steps: int, start_step: int = 0):
        step = start_step
        it = iter(dataloader)
        while step < total_steps:
            mbs = []
            for _ in range(self.grad_accum_steps):
                try:
                    b = next(it)
                except StopIteration:
                    it = iter(dataloader)
                    b = next(it)
                mbs.append({k: v.to(self.device, non_blocking=True) for k, v in b.items()})
            out = self.engine.train_step(mbs)
            step += 1
            if step % self.logger.log_interval == 0:
                self.logger.log_step(step=step, loss=out["loss"],
                                     lr=self.scheduler.get_last_lr()[0],
                                     grad_norm=out["grad_norm"])
            if self.ckpt_mgr.should_save(step):
                m, o, s = self.engine.state_for_save()
                self.ckpt_mgr.save(step, m, o, s, extra_state={"step": step})
        self.ckpt_mgr.wait()
        self.logger.finish()


class ThinkingModeFusion:
    """Mix thinking and non-thinking samples (reference: training/sft.py:255-306).

    Non-thinking samples get an empty reasoning block.  ``thinking_ratio`` is
    the fraction of thinking samples in the mix.
    """

    def __init__(self, thinking_ratio: float = 0.5, system_prompt: str = "You are a helpful assistant.",
                 seed: int = 0):
        self.thinking_ratio = thinking_ratio
        self.system_prompt = system_prompt
        self.seed = seed

    def prepare_dataset(self, thinking_samples: List[Dict], non_thinking_samples: List[Dict]) -> List[Dict]:
        nt = []
        for s in non_thinking_samples:
            convs = [dict(t, reasoning=t.get("reasoning", "")) for t in s.get("conversations", [])]
            nt.append(dict(s, conversations=convs))
        r = min(max(self.thinking_ratio, 0.0), 0.999)
        n_think = min(len(thinking_samples), int(round(len(nt) * r / (1 - r))))
        mixed = list(thinking_samples[:n_think]) + nt
        random.Random(self.seed).shuffle(mixed)
        return mixed


DUMMY_SFT = [{"conversations": [{"user": "What is 2+2?", "assistant": "4", "reasoning": "2+2=4"}]}]


def run_sft(model_config_path: str, training_config_path: str, variant: str = "cold_start",
            resume_from: Optional[str] = None, max_samples: Optional[int] = None,
            max_steps: Optional[int] = None):
    rank, world = init_distributed()
    device = pick_device()
    mcfg = ModelConfig.from_yaml(model_config_path)
    with open(training_config_path) as f:
        tcfg = yaml.safe_load(f) or {}
    torch.manual_seed(tcfg.get("seed", 0))
    model = Qwen3Model(mcfg)
    if is_main_process():
        print(f"SFT | params: {model.count_parameters()['total']:,} | variant: {variant}")
    bcfg = tcfg.get("batch", {}) or {}
    scfg = tcfg.get("sft", {}) or {}
    S = bcfg.get("max_seq_len", 8192)
    tok = Tokenizer(backend="auto")
    kw = dict(mask_input=scfg.get("mask_input", True),
              thinking_enabled=scfg.get("thinking_enabled", True),
              think_open=scfg.get("think_token", "<think>"),
              think_close=scfg.get("no_think_token", "</think>"))
    try:
        from ..data.hf_datasets import load_sft_dataset
        ds = load_sft_dataset(variant, tok, S, max_samples, kw["thinking_enabled"])
        ds.mask_input, ds.think_open, ds.think_close = kw["mask_input"], kw["think_open"], kw["think_close"]
    except Exception as exc:
        if is_main_process():
            print(f"HF dataset load failed ({type(exc).__name__}), falling back to dummy data")
        ds = SFTDataset(DUMMY_SFT * 100, tok, S, **kw)
    # the same model-parallel layouts as pretraining; one data shard per
    # data-parallel rank
    from .pretrain import build_parallel
    parallel = build_parallel(tcfg, world)
    dp_rank, dp_size = rank, world
    if parallel is not None:
        model = parallel.apply_parallelism(model.to(device))
        dp_rank, dp_size = parallel.coords["dp"], parallel.config.dp_size
    sampler = DistributedSampler(ds, num_replicas=dp_size, rank=dp_rank)
    loader = DataLoader(ds, batch_size=bcfg.get("micro_batch_size", 2), sampler=sampler,
                        collate_fn=TextCollator(), num_workers=0)
    trainer = SFTTrainer(model, tcfg, device, parallel=parallel)
    start = 0
    resume_from = resolve_resume(resume_from, tcfg, trainer.ckpt_mgr)
    if resume_from:
        start = int(trainer.ckpt_mgr.load(trainer.model, trainer.optimizer, trainer.scheduler,
                                          resume_from).get("step", 0))
    total = max_steps or (tcfg.get("scheduler", {}) or {}).get("total_steps", 5000)
    trainer.train(loader, total, start)
    return trainer
