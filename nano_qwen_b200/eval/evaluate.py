"""Evaluation harness: perplexity, multiple choice and generative accuracy.

Same methods and result dictionaries as the reference's ``Evaluator``
(reference: eval/evaluate.py:18-147).  Perplexity and choice scoring use the
fused lm_head + cross-entropy kernel (per-token log-probs without [T, V]
logits); multiple-choice scores every choice of a question in one batched
forward; generative evaluation uses the KV-cache generator.
"""

from __future__ import annotations

import math
from typing import Dict, List, Optional

import torch

from .. import ops
from ..models.transformer import shift_targets
from .generate import TextGenerator


class Evaluator:
    def __init__(self, model, tokenizer, device: torch.device = torch.device("cpu")):
        self.model = model
        self.tokenizer = tokenizer
        self.device = device
        self.generator = TextGenerator(model, tokenizer, device)

    @torch.no_grad()
    def compute_perplexity(self, eval_dataloader, max_batches: Optional[int] = None) -> float:
        self.model.eval()
        total_nll, total_tok, n = 0.0, 0, 0
        for batch in eval_dataloader:
            ids = batch["input_ids"].to(self.device)
            labels = batch["labels"].to(self.device)
            x, _, _ = self.model.hidden(ids)
            tgt = shift_targets(labels)
            nll = ops.linear_cross_entropy(x, self.model.lm_head_ref(x.dtype), tgt, reduction="none")
            valid = (tgt != -100)
            total_nll += float(nll[valid].sum())
            total_tok += int(valid.sum())
            n += 1
            if max_batches and n >= max_batches:
                break
        return math.exp(total_nll / max(total_tok, 1))

    @torch.no_grad()
    def choice_logprob(self, prompt: str, choices: List[str]) -> List[float]:
        """Mean log-prob of each choice's tokens given the prompt (reference scoring)."""
        enc = lambda s: self.tokenizer.encode(s, allowed_special="all")
        p_ids = enc(prompt)
        seqs = [enc(prompt + " " + c) for c in choices]
        L = max(len(s) for s in seqs)
        pad = 0
        ids = torch.full((len(seqs), L), pad, dtype=torch.long)
        tgt = torch.full((len(seqs), L), -100, dtype=torch.long)
        for i, s in enumerate(seqs):
            ids[i, :len(s)] = torch.tensor(s)
            # position t predicts token t+1; score only the choice tokens
            for t in range(len(p_ids) - 1, len(s) - 1):
                tgt[i, t] = s[t + 1]
        ids, tgt = ids.to(self.device), tgt.to(self.device)
        x, _, _ = self.model.hidden(ids)
        nll = ops.linear_cross_entropy(x, self.model.lm_head_ref(x.dtype), tgt, reduction="none")
        out = []
        for i in range(len(seqs)):
            m = tgt[i] != -100
            out.append(float(-(nll[i][m]).mean()) if bool(m.any()) else float("-inf"))
        return out

    def eval_multiple_choice(self, questions: List[Dict], num_choices: int = 4) -> dict:
        self.model.eval()
        correct = 0
        for q in questions:
            scores = self.choice_logprob(q["prompt"], q["choices"])
            pred = max(range(len(scores)), key=lambda i: scores[i])
            correct += int(pred == q["answer"])
        total = len(questions)
        return {"accuracy": correct / max(total, 1), "correct": correct, "total": total}

    def eval_generative(self, questions: List[Dict], metric_fn=None,
                        max_new_tokens: int = 512) -> dict:
        preds, refs = [], []
        for q in questions:
            preds.append(self.generator.generate(q["prompt"], max_new_tokens=max_new_tokens,
                                                 temperature=0.0))
            refs.append(q["answer"])
        if metric_fn is not None:
            return metric_fn(preds, refs)
        correct = sum(1 for p, r in zip(preds, refs) if r.strip() in p)
        return {"accuracy": correct / max(len(preds), 1), "correct": correct, "total": len(preds)}
