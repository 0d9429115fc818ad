"""Group Relative Policy Optimization.

Same algorithm and surface as the reference (``GRPO.generate_responses /
compute_advantages / compute_kl_penalty / policy_loss / train_step / train``,
``_math_reward_fn``, ``run_grpo``; reference: training/grpo.py:31-400): sample
G responses per prompt, reward them, advantages (r - mean) / std, per-token
clipped surrogate plus a KL term against a frozen reference copy.

Differences: rollouts use the KV-cache generator (one decode step per token,
CUDA-graph replayed on GPU; the reference re-ran the full sequence per token);
old and new log-probs are both taken from the temperature-scaled distribution
(the reference mixed scaled and unscaled logits, training/grpo.py:100 vs
:172-173); tokens after the first EOS are masked out of the loss; log-probs
come from the fused lm_head + CE kernel.
"""

from __future__ import annotations

import copy
import re
from typing import Callable, List, Optional, Tuple

import torch

from .. import ops
from .checkpoint import manager_from_config, resolve_resume
from .engine import TrainEngine


def response_logprobs(model, seqs: torch.Tensor, prompt_len: int, temperature: float) -> torch.Tensor:
    """log p(seqs[:, t] | seqs[:, <t]) for the response tokens t >= prompt_len: [B, T_resp]."""
    x, _, _ = model.hidden(seqs)
    B, L = seqs.shape
    tgt = torch.full_like(seqs, -100)
    tgt[:, prompt_len - 1:L - 1] = seqs[:, prompt_len:]
    lp = ops.token_logprobs(x, model.lm_head_ref(x.dtype), tgt, temperature=temperature)
    return lp[:, prompt_len - 1:L - 1]


class GRPO:
    def __init__(self, policy_model, ref_model, tokenizer, config: dict, device: torch.device):
        g = config.get("grpo", {}) or {}
        self.group_size = g.get("group_size", 16)
        self.clip_ratio = g.get("clip_ratio", 0.2)
        self.kl_coef = g.get("kl_coef", 0.01)
        self.temperature = g.get("temperature", 0.7)
        self.max_gen_len = g.get("max_gen_len", 2048)
        self.tokenizer = tokenizer
        self.device = device
        cfg = dict(config)
        cfg.setdefault("optimizer", {"lr": 5e-7})
        sch = dict(cfg.get("scheduler", {}) or {})
        sch.setdefault("warmup_steps", 50)
        sch.setdefault("total_steps", 2000)
        cfg["scheduler"] = sch
        self.engine = TrainEngine(policy_model, cfg, device)
        self.policy = self.engine.model
        self.optimizer = self.engine.optimizer
        self.scheduler = self.engine.scheduler
        self.ref = ref_model.to(device) if ref_model is not None else None
        if self.ref is not None:
            self.ref.eval()
            for p in self.ref.parameters():
                p.requires_grad_(False)
        self.last_metrics: dict = {}

    @torch.no_grad()
    def generate_responses(self, prompt_ids: torch.Tensor, num_samples: int):
        """(sequences [G, P+T], old log-probs [G, T], response mask [G, T])."""
        from ..eval.generate import TextGenerator
        gen = TextGenerator(self.policy, self.tokenizer, self.device)
        prompt = prompt_ids.expand(num_samples, -1).to(self.device)
        toks, lps, mask = gen.sample_batch(prompt, self.max_gen_len, self.temperature,
                                           eos_id=getattr(self.tokenizer, "eos_id", None))
        self.policy.train()
        return torch.cat([prompt, toks], 1), lps, mask

    @staticmethod
    def compute_advantages(rewards: torch.Tensor) -> torch.Tensor:
        return (rewards - rewards.mean()) / rewards.std().clamp(min=1e-8)

    def compute_kl_penalty(self, seqs, prompt_len, policy_lp, mask) -> torch.Tensor:
        if self.ref is None:
            return torch.zeros(seqs.shape[0], device=self.device)
        with torch.no_grad():
            ref_lp = response_logprobs(self.ref, seqs, prompt_len, self.temperature)
        m = mask.float()
        return ((policy_lp - ref_lp) * m).sum(1) / m.sum(1).clamp(min=1)

    def policy_loss(self, seqs, prompt_len, old_lp, advantages, mask) -> Tuple[torch.Tensor, dict]:
        new_lp = response_logprobs(self.policy, seqs, prompt_len, self.temperature)
        ratio = torch.exp(new_lp - old_lp)
        adv = advantages.unsqueeze(1).expand_as(ratio)
        surr = torch.min(ratio * adv, ratio.clamp(1 - self.clip_ratio, 1 + self.clip_ratio) * adv)
        m = mask.float()
        pl = -(surr * m).sum() / m.sum().clamp(min=1)
        kl = self.compute_kl_penalty(seqs, prompt_len, new_lp, mask)
        total = pl + self.kl_coef * kl.mean()
        return total, {"policy_loss": pl.detach(), "kl": kl.mean().detach(),
                       "ratio_mean": (ratio * m).sum().detach() / m.sum().clamp(min=1),
                       "advantages_mean": advantages.mean()}

    def train_step(self, prompt_ids: torch.Tensor, reward_fn: Callable,
                   ground_truth: Optional[str] = None, prompt: Optional[str] = None) -> dict:
        seqs, old_lp, mask = self.generate_responses(prompt_ids, self.group_size)
        P = prompt_ids.shape[1]
        texts = [self.tokenizer.decode(s[P:][m].tolist()) for s, m in zip(seqs, mask)]
        if hasattr(reward_fn, "set_prompt"):
            reward_fn.set_prompt(prompt if prompt is not None else self.tokenizer.decode(
                prompt_ids[0].tolist()))
        rewards = reward_fn(texts, ground_truth)
        rewards = torch.as_tensor(rewards, dtype=torch.float32, device=self.device)
        adv = self.compute_advantages(rewards)

        def loss_fn(model, mb):
            loss, m = self.policy_loss(seqs, P, old_lp, adv, mask)
            self.last_metrics = m
            return loss

        out = self.engine.train_step([{}], loss_fn=loss_fn)
        metrics = {k: float(v) for k, v in self.last_metrics.items()}
        metrics.update(reward_mean=float(rewards.mean()), reward_std=float(rewards.std()),
                       total_loss=float(out["loss"]), grad_norm=float(out["grad_norm"]))
        return metrics

    def train(self, queries: List[dict], reward_fn: Callable, total_steps: int, start_step: int = 0,
              ckpt_mgr=None):
        """Steps ``start_step + 1 .. total_steps`` (one prompt each, cycling
        through ``queries``); checkpoints every ``save_interval`` steps when a
        manager is given."""
        from .logger import TrainingLogger
        logger = TrainingLogger(log_interval=1)
        for step in range(start_step, total_steps):
            q = queries[step % len(queries)]
            ids = torch.tensor(self.tokenizer.encode(q["prompt"]), dtype=torch.long).unsqueeze(0)
            m = self.train_step(ids, reward_fn, q.get("answer"), q["prompt"])
            logger.log_step(step=step + 1, loss=m["total_loss"], lr=self.scheduler.get_last_lr()[0],
                            grad_norm=m["grad_norm"], extra={f"rl/{k}": v for k, v in m.items()})
            if ckpt_mgr is not None and ckpt_mgr.should_save(step + 1):
                mdl, opt, sch = self.engine.state_for_save()
                ckpt_mgr.save(step + 1, mdl, opt, sch, extra_state={"step": step + 1})
        if ckpt_mgr is not None:
            ckpt_mgr.wait()
        logger.finish()


def _extract_answer(text: str) -> str:
    boxed = re.findall(r"\\boxed\{([^}]+)\}", text)
    if boxed:
        return boxed[-1].strip()
    hashes = re.findall(r"####\s*(.+)", text)
    if hashes:
        return hashes[-1].strip()
    nums = re.findall(r"-?\d+\.?\d*", text)
    return nums[-1] if nums else ""


def _math_reward_fn(responses: List[str], ground_truth: Optional[str]) -> List[float]:
    """1.0 when the final answer (\\boxed{}, '####' or last number) matches
    (reference: training/grpo.py:288-312)."""
    if ground_truth is None:
        return [0.0] * len(responses)
    gt = _extract_answer(ground_truth)
    out = []
    for r in responses:
        p = _extract_answer(r)
        try:
            out.append(1.0 if abs(float(p) - float(gt)) < 1e-6 else 0.0)
        except (ValueError, ZeroDivisionError):
            out.append(1.0 if p == gt else 0.0)
    return out


class CombinedReward:
    """Weighted sum of the reward sources a training YAML's
    ``grpo.reward_types`` names (the reference lists them but always uses
    the math reward):

    * ``verifiable``: 1.0 when the final answer matches the ground truth;
    * ``model``: a trained ``RewardModel`` (``grpo.reward_model_checkpoint``,
      a ``checkpoint.pt`` with its state dict; model shape from the policy's
      config) scoring prompt + response.

    ``grpo.reward_weights`` (same order, default 1.0 each) weights them."""

    def __init__(self, fns: List[Tuple[str, Callable, float]]):
        self.fns = fns
        self.prompt = ""

    def set_prompt(self, prompt: str) -> None:
        self.prompt = prompt

    def __call__(self, responses: List[str], ground_truth: Optional[str]) -> List[float]:
        total = [0.0] * len(responses)
        for _, fn, w in self.fns:
            vals = fn(responses, ground_truth, self.prompt)
            total = [t + w * float(v) for t, v in zip(total, vals)]
        return total


def build_reward_fn(training_config: dict, model_config=None, tokenizer=None,
                    device: torch.device = torch.device("cpu")) -> CombinedReward:
    g = training_config.get("grpo", {}) or {}
    types = list(g.get("reward_types") or ["verifiable"])
    weights = list(g.get("reward_weights") or [1.0] * len(types))
    if len(weights) != len(types):
        raise ValueError("grpo.reward_weights needs one weight per reward type")
    fns: List[Tuple[str, Callable, float]] = []
    for kind, w in zip(types, weights):
        if kind == "verifiable":
            fns.append((kind, lambda r, gt, prompt: _math_reward_fn(r, gt), float(w)))
        elif kind == "model":
            path = g.get("reward_model_checkpoint")
            if not path:
                from ..parallel.comm import is_main_process
                if is_main_process():
                    print("grpo.reward_types lists 'model' but grpo.reward_model_checkpoint is "
                          "not set: the model reward is skipped")
                continue
            fns.append((kind, _model_reward(path, model_config, tokenizer, device), float(w)))
        else:
            raise ValueError(f"unknown reward type {kind!r} (verifiable, model)")
    if not fns:
        raise ValueError("no usable reward in grpo.reward_types")
    return CombinedReward(fns)


def _model_reward(path: str, model_config, tokenizer, device):
    from .reward_model import RewardModel
    rm = RewardModel(model_config)
    st = torch.load(path, map_location="cpu", weights_only=False)
    rm.load_state_dict(st.get("model", st))
    rm = rm.to(device).eval()

    @torch.no_grad()
    def score(responses, ground_truth, prompt):
        seqs = [tokenizer.encode(prompt + r) for r in responses]
        L = max(len(x) for x in seqs)
        ids = torch.zeros(len(seqs), L, dtype=torch.long)
        mask = torch.zeros(len(seqs), L, dtype=torch.long)
        for i, x in enumerate(seqs):
            ids[i, :len(x)] = torch.tensor(x, dtype=torch.long)
            mask[i, :len(x)] = 1
        return rm(ids.to(device), mask.to(device)).float().cpu().tolist()
    return score


def run_grpo(model_config_path: str, training_config_path: str, resume_from: Optional[str] = None,
             max_samples: Optional[int] = None, max_steps: Optional[int] = None):
    import yaml

    from ..config import ModelConfig
    from ..data.tokenizer import Tokenizer
    from ..models.transformer import Qwen3Model
    from ..parallel.comm import init_distributed, is_main_process
    from .pretrain import pick_device

    init_distributed()
    device = pick_device()
    mcfg = ModelConfig.from_yaml(model_config_path)
    with open(training_config_path) as f:
        tcfg = yaml.safe_load(f) or {}
    torch.manual_seed(tcfg.get("seed", 0))
    policy = Qwen3Model(mcfg)
    ref = copy.deepcopy(policy)
    tok = Tokenizer(backend="auto")
    try:
        from ..data.hf_datasets import load_grpo_dataset
        queries = load_grpo_dataset(max_samples=max_samples)
    except Exception as exc:
        if is_main_process():
            print(f"HF dataset load failed ({type(exc).__name__}), using dummy queries")
        queries = [{"prompt": "What is 15 + 27?", "answer": "42"},
                   {"prompt": "What is 100 - 37?", "answer": "63"}] * 50
    trainer = GRPO(policy, ref, tok, tcfg, device)
    mgr = manager_from_config(tcfg, "checkpoints/rl")
    start = 0
    resume_from = resolve_resume(resume_from, tcfg, mgr)
    if resume_from:
        start = int(mgr.load(trainer.policy, trainer.optimizer, trainer.scheduler,
                             resume_from).get("step", 0))
    total = max_steps or (tcfg.get("scheduler", {}) or {}).get("total_steps", 2000)
    reward = build_reward_fn(tcfg, mcfg, tok, device)
    trainer.train(queries, reward, total, start, mgr)
    return trainer
