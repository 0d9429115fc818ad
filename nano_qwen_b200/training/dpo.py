"""Direct Preference Optimization (offline and online).

Same trainer surface as the reference (``DPOTrainer.dpo_loss / train_step``,
``OnlineDPO.generate_preference_pair / online_train_step``, ``run_dpo``;
reference: training/dpo.py:25-328): sequence score = mean per-token
log-prob of the label tokens, loss = -logsigmoid(beta * delta) with optional
label smoothing and a reference-free mode.  Per-token log-probs come from the
fused lm_head + cross-entropy kernel (no [B, S, V] log-softmax), chosen and
rejected sequences run as one batch, and online DPO samples candidates with the
KV-cache generator (the reference re-ran the full sequence for every token).
"""

from __future__ import annotations

import copy
from typing import Callable, Optional, Tuple

import torch
import torch.nn.functional as F

from .. import ops
from ..models.transformer import shift_targets
from .checkpoint import manager_from_config, resolve_resume
from .engine import TrainEngine


def sequence_logprobs(model, ids: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
    """Mean log p(label_{t+1} | <= t) over valid targets, per sequence [B]."""
    x, _, _ = model.hidden(ids)
    tgt = shift_targets(labels)
    lp = -ops.linear_cross_entropy(x, model.lm_head_ref(x.dtype), tgt, reduction="none")
    m = (tgt != -100).float()
    return (lp * m).sum(-1) / m.sum(-1).clamp(min=1.0)


class DPOTrainer:
    def __init__(self, policy_model, ref_model, config: dict, device: torch.device, dp_group=None):
        """``dp_group``: the data-parallel ranks (default: every rank)."""
        dcfg = config.get("dpo", {}) or {}
        self.beta = dcfg.get("beta", 0.1)
        self.label_smoothing = dcfg.get("label_smoothing", 0.0)
        self.reference_free = dcfg.get("reference_free", False)
        self.device = device
        cfg = dict(config)
        cfg.setdefault("optimizer", {"lr": 5e-7})
        sch = dict(cfg.get("scheduler", {}) or {})
        sch.setdefault("warmup_steps", 50)
        sch.setdefault("total_steps", 2000)
        cfg["scheduler"] = sch
        self.engine = TrainEngine(policy_model, cfg, device, dp_group=dp_group)
        self.policy = self.engine.model
        self.optimizer = self.engine.optimizer
        self.scheduler = self.engine.scheduler
        self.ref = ref_model.to(device) if ref_model is not None else None
        if self.ref is not None:
            self.ref.eval()
            for p in self.ref.parameters():
                p.requires_grad_(False)
        self.grad_clip = self.engine.grad_clip
        self.last_metrics: dict = {}

    def dpo_loss(self, chosen_ids, rejected_ids, chosen_labels, rejected_labels) -> Tuple[torch.Tensor, dict]:
        ids = torch.cat([chosen_ids, rejected_ids], 0)
        labels = torch.cat([chosen_labels, rejected_labels], 0)
        n = chosen_ids.shape[0]
        pi = sequence_logprobs(self.policy, ids, labels)
        with torch.no_grad():
            if self.reference_free or self.ref is None:
                rf = torch.zeros_like(pi)
            else:
                rf = sequence_logprobs(self.ref, ids, labels)
        lc = pi[:n] - rf[:n]
        lr = pi[n:] - rf[n:]
        logits = self.beta * (lc - lr)
        if self.label_smoothing > 0:
            loss = (-F.logsigmoid(logits) * (1 - self.label_smoothing)
                    - F.logsigmoid(-logits) * self.label_smoothing).mean()
        else:
            loss = -F.logsigmoid(logits).mean()
        cr, rr = self.beta * lc.detach(), self.beta * lr.detach()
        metrics = {"loss": loss.detach(), "accuracy": (logits > 0).float().mean().detach(),
                   "chosen_rewards": cr.mean(), "rejected_rewards": rr.mean(),
                   "reward_margin": (cr - rr).mean()}
        return loss, metrics

    def train_step(self, chosen_ids, rejected_ids, chosen_labels, rejected_labels) -> dict:
        batch = {k: v.to(self.device) for k, v in dict(c=chosen_ids, r=rejected_ids,
                                                         cl=chosen_labels, rl=rejected_labels).items()}

        def loss_fn(model, mb):
            loss, m = self.dpo_loss(mb["c"], mb["r"], mb["cl"], mb["rl"])
            self.last_metrics = m
            return loss

        out = self.engine.train_step([batch], loss_fn=loss_fn)
        metrics = {k: float(v) for k, v in self.last_metrics.items()}
        metrics["grad_norm"] = float(out["grad_norm"])
        return metrics


class OnlineDPO(DPOTrainer):
    """Sample candidates from the current policy, rank them with a reward
    function, train on (best, worst) (reference: training/dpo.py:167-223)."""

    def __init__(self, policy_model, ref_model, reward_fn: Callable, tokenizer, config: dict,
                 device: torch.device, max_new_tokens: int = 512, temperature: float = 0.7):
        super().__init__(policy_model, ref_model, config, device)
        self.reward_fn = reward_fn
        self.tokenizer = tokenizer
        self.num_candidates = (config.get("grpo", {}) or {}).get("group_size", 4)
        self.max_new_tokens = max_new_tokens
        self.temperature = temperature

    @torch.no_grad()
    def generate_preference_pair(self, prompt_ids: torch.Tensor):
        from ..eval.generate import TextGenerator
        gen = TextGenerator(self.policy, self.tokenizer, self.device)
        prompt = prompt_ids.expand(self.num_candidates, -1).to(self.device)
        toks, _, mask = gen.sample_batch(prompt, self.max_new_tokens, self.temperature,
                                         eos_id=getattr(self.tokenizer, "eos_id", None))
        self.policy.train()
        seqs = torch.cat([prompt, toks], 1)
        texts = [self.tokenizer.decode(s[m].tolist()) for s, m in
                 zip(seqs, torch.cat([torch.ones_like(prompt, dtype=torch.bool), mask], 1))]
        rewards = self.reward_fn(texts)
        if not isinstance(rewards, torch.Tensor):
            rewards = torch.tensor(rewards, dtype=torch.float32)
        b, w = int(rewards.argmax()), int(rewards.argmin())
        return seqs[b:b + 1], seqs[w:w + 1]

    def online_train_step(self, prompt_ids: torch.Tensor) -> dict:
        chosen, rejected = self.generate_preference_pair(prompt_ids)
        return self.train_step(chosen, rejected, chosen, rejected)


def run_dpo(model_config_path: str, training_config_path: str, resume_from: Optional[str] = None,
            max_samples: Optional[int] = None, max_steps: Optional[int] = None):
    import yaml
    from torch.utils.data import DataLoader

    from ..config import ModelConfig
    from ..data.hf_datasets import DPODataset
    from ..data.sampler import DistributedSampler
    from ..data.tokenizer import Tokenizer
    from ..models.transformer import Qwen3Model
    from ..parallel.comm import init_distributed, is_main_process
    from .logger import TrainingLogger
    from .pretrain import pick_device

    rank, world = init_distributed()
    device = pick_device()
    mcfg = ModelConfig.from_yaml(model_config_path)
    with open(training_config_path) as f:
        tcfg = yaml.safe_load(f) or {}
    torch.manual_seed(tcfg.get("seed", 0))
    policy = Qwen3Model(mcfg)
    ref = copy.deepcopy(policy)
    tok = Tokenizer(backend="auto")
    S = (tcfg.get("batch", {}) or {}).get("max_seq_len", 2048)
    try:
        from ..data.hf_datasets import load_dpo_dataset
        ds = load_dpo_dataset(tok, S, max_samples=max_samples)
    except Exception as exc:
        if is_main_process():
            print(f"HF dataset load failed ({type(exc).__name__}), using dummy pairs")
        ds = DPODataset([{"prompt": "User: Hi\nAssistant: ",
                          "chosen": "User: Hi\nAssistant: Hello! How can I help?",
                          "rejected": "User: Hi\nAssistant: What do you want?"}] * 100, tok, S)
    if is_main_process():
        print(f"DPO | params: {policy.count_parameters()['total']:,} | pairs: {len(ds)}")
    sampler = DistributedSampler(ds, num_replicas=world, rank=rank)
    loader = DataLoader(ds, batch_size=(tcfg.get("batch", {}) or {}).get("micro_batch_size", 2),
                        sampler=sampler, num_workers=0)
    trainer = DPOTrainer(policy, ref, tcfg, device)
    mgr = manager_from_config(tcfg, "checkpoints/dpo")
    start = 0
    resume_from = resolve_resume(resume_from, tcfg, mgr)
    if resume_from:
        start = int(mgr.load(trainer.policy, trainer.optimizer, trainer.scheduler, resume_from,
                             sampler=sampler).get("step", 0))
    logger = TrainingLogger(log_interval=1)
    total = max_steps or (tcfg.get("scheduler", {}) or {}).get("total_steps", 2000)
    it = iter(loader)
    for step in range(start + 1, total + 1):
        try:
            b = next(it)
        except StopIteration:
            it = iter(loader)
            b = next(it)
        m = trainer.train_step(b["chosen_ids"], b["rejected_ids"], b["chosen_labels"], b["rejected_labels"])
        logger.log_step(step=step, loss=m["loss"], lr=trainer.scheduler.get_last_lr()[0],
                        grad_norm=m["grad_norm"], extra={f"dpo/{k}": v for k, v in m.items()})
        if mgr.should_save(step):
            mdl, opt, sch = trainer.engine.state_for_save()
            mgr.save(step, mdl, opt, sch, extra_state={"step": step}, sampler=sampler)
    mgr.wait()
    logger.finish()
    return trainer
