"""CPU tests of the model, config, optimizer, scheduler and checkpointing
against the reference implementation (imported read-only from
``baseline/_ref``) and against plain PyTorch."""

import math
import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")
HAS_REF = os.path.isdir(os.path.join(REF, "model"))


def _ref_import():
    if REF not in sys.path:
        sys.path.append(REF)
    from model.config import ModelConfig as RC
    from model.transformer import Qwen3Model as RM
    return RC, RM


TINY = dict(hidden_size=64, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
            head_dim=16, intermediate_size=128, vocab_size=256, max_position_embeddings=128,
            tie_word_embeddings=True)
TINY_MOE = dict(TINY, num_experts=4, num_experts_per_tok=2, moe_intermediate_size=32,
                tie_word_embeddings=False)


# ------------------------------------------------------------------ config
def test_config_defaults_and_yaml():
    from nano_qwen_b200.config import PRESETS, ModelConfig
    c = ModelConfig()
    assert c.head_dim == c.hidden_size // c.num_attention_heads
    for name in ("debug", "small", "medium", "large"):
        y = ModelConfig.from_yaml(os.path.join(ROOT, "configs", "model", f"{name}.yaml"))
        assert y.hidden_size > 0 and y.num_hidden_layers > 0
    assert "debug" in PRESETS
    m = ModelConfig(**TINY_MOE)
    assert m.layer_is_moe(0) and m.active_params_per_token() < m.total_params_estimate()


@pytest.mark.skipif(not HAS_REF, reason="reference copy not present")
@pytest.mark.parametrize("cfg", [TINY, TINY_MOE])
def test_model_matches_reference(cfg):
    RC, RM = _ref_import()
    from nano_qwen_b200.config import ModelConfig
    from nano_qwen_b200.models import Qwen3Model
    torch.manual_seed(0)
    ref = RM(RC(**cfg))
    ours = Qwen3Model(ModelConfig(**cfg))
    ours.load_state_dict(ref.state_dict())
    ids = torch.randint(0, cfg["vocab_size"], (2, 24))
    a = ref(input_ids=ids, labels=ids)
    b = ours(ids, labels=ids)
    assert torch.allclose(a["loss"], b["loss"], atol=1e-5, rtol=1e-5)
    a["loss"].backward()
    b["loss"].backward()
    rp = dict(ref.named_parameters())
    for n, p in ours.named_parameters():
        assert torch.allclose(p.grad, rp[n].grad, atol=1e-5, rtol=1e-4), n
    la = ref(input_ids=ids)["logits"]
    lb = ours(ids)["logits"]
    assert torch.allclose(la, lb, atol=1e-5, rtol=1e-5)


def test_kv_cache_decode_matches_full_forward():
    from nano_qwen_b200.config import ModelConfig
    from nano_qwen_b200.models import Qwen3Model
    from nano_qwen_b200.models.kv_cache import KVCache
    torch.manual_seed(0)
    cfg = ModelConfig(**TINY)
    m = Qwen3Model(cfg).eval()
    ids = torch.randint(0, 256, (2, 12))
    with torch.no_grad():
        full = m(ids)["logits"]
        caches = [KVCache() for _ in range(cfg.num_hidden_layers)]
        a = m(ids[:, :8], kv_caches=caches)["logits"]
        steps = [a]
        for t in range(8, 12):
            steps.append(m(ids[:, t:t + 1], kv_caches=caches)["logits"])
    inc = torch.cat(steps, 1)
    assert torch.allclose(inc, full, atol=1e-4, rtol=1e-4)


def test_yarn_rope_tables():
    from nano_qwen_b200.models.rope import rope_tables
    cos, sin = rope_tables(64, 128, 1e6, {"type": "yarn", "factor": 4.0,
                                         "original_max_position_embeddings": 32})
    assert cos.shape == (128, 32) and torch.isfinite(cos).all() and torch.isfinite(sin).all()
    c0, _ = rope_tables(64, 128, 1e6, None)
    assert not torch.allclose(cos, c0)


# ------------------------------------------------------------------ optimizer
def test_fused_adamw_cpu_matches_torch():
    from nano_qwen_b200.config import ModelConfig
    from nano_qwen_b200.models import Qwen3Model
    from nano_qwen_b200.training.optimizer import attach_param_store, build_optimizer
    torch.manual_seed(0)
    cfg = ModelConfig(**TINY)
    a = Qwen3Model(cfg)
    b = Qwen3Model(cfg)
    b.load_state_dict(a.state_dict())
    store = attach_param_store(a, torch.float32, torch.device("cpu"))
    opt_a = build_optimizer(a, lr=1e-2, weight_decay=0.1, fused=True, store=store)
    decay = [p for n, p in b.named_parameters()
             if not (p.ndim <= 1 or "norm" in n or "bias" in n or "embed" in n)]
    nodecay = [p for n, p in b.named_parameters()
               if (p.ndim <= 1 or "norm" in n or "bias" in n or "embed" in n)]
    opt_b = torch.optim.AdamW([{"params": decay, "weight_decay": 0.1},
                               {"params": nodecay, "weight_decay": 0.0}],
                              lr=1e-2, betas=(0.9, 0.95), eps=1e-8)
    ids = torch.randint(0, 256, (2, 16))
    for _ in range(3):
        store.zero_grad()
        a(ids, labels=ids)["loss"].backward()
        opt_a.clip_grad_norm_(0.0)
        opt_a.step()
        opt_b.zero_grad()
        b(ids, labels=ids)["loss"].backward()
        opt_b.step()
    bp = dict(b.named_parameters())
    for n, p in a.named_parameters():
        assert torch.allclose(p, bp[n], atol=1e-5, rtol=1e-4), n


def test_fused_adamw_pieces_match_whole_store():
    """Moments kept for a list of flat ranges (back to back): three
    optimizers whose pieces cover the store between them update exactly like
    one whole-store optimizer, and their gathered moments agree."""
    from nano_qwen_b200.config import ModelConfig
    from nano_qwen_b200.models import Qwen3Model
    from nano_qwen_b200.training.optimizer import FusedAdamW, attach_param_store
    torch.manual_seed(0)
    cfg = ModelConfig(**TINY)
    a = Qwen3Model(cfg)
    store = attach_param_store(a, torch.float32, torch.device("cpu"))
    n = store.numel
    cut = [0, n // 64 // 3 * 64, 2 * n // 64 // 3 * 64, n]
    whole = FusedAdamW(store, lr=1e-2, weight_decay=0.1)
    parts = [[(cut[0], cut[1]), (cut[2], cut[3])], [(cut[1], cut[2])]]
    opts = [FusedAdamW(store, lr=1e-2, weight_decay=0.1, pieces=pc) for pc in parts]
    assert [o.exp_avg.numel() for o in opts] == [cut[1] + n - cut[2], cut[2] - cut[1]]
    ids = torch.randint(0, 256, (2, 16))
    start = store.master.clone()
    store.zero_grad()
    a(ids, labels=ids)["loss"].backward()
    # the pieces' squared norms add up to the whole store's
    sq = sum(float(o.clip_grad_norm_(0.0)) ** 2 for o in opts)
    assert abs(sq - float(whole.clip_grad_norm_(0.0)) ** 2) < 1e-5 * sq
    for _ in range(2):
        whole.step()
    ref = store.master.clone()
    store.master.copy_(start)
    for _ in range(2):
        for o in opts:
            o.step()
    assert torch.allclose(store.master, ref, atol=1e-6, rtol=1e-5)
    full = torch.zeros(n)
    for o in opts:
        o.gather_full_state()
        for p in store.params:
            full_view = o.state[p]["exp_avg"]
            o_ = store.offset(p)
            full[o_:o_ + p.numel()] += full_view.reshape(-1)
    assert torch.allclose(full, whole.exp_avg, atol=1e-7)


def test_flat_store_pads_expert_span_to_shard_multiple():
    """The expert span starts and ends on a multiple of pad_multiple, so the
    dense pieces around it and the span itself split into equal shards."""
    from nano_qwen_b200.config import ModelConfig
    from nano_qwen_b200.models import Qwen3Model
    from nano_qwen_b200.training.optimizer import attach_param_store
    torch.manual_seed(0)
    cfg = ModelConfig(**dict(TINY, num_experts=4, num_experts_per_tok=2, moe_intermediate_size=32))
    m = Qwen3Model(cfg)
    for n, p in m.named_parameters():
        if ".experts." in n:
            p._ep_local = True
    store = attach_param_store(m, torch.float32, torch.device("cpu"), pad_multiple=64 * 8)
    xb, xe = store.expert_span
    assert xe > xb and xb % 512 == 0 and xe % 512 == 0 and store.numel % 512 == 0
    for n, p in zip(store.names, store.params):
        o = store.offset(p)
        inside = xb <= o < xe
        assert inside == (".experts." in n), n


def test_grad_clip_norm():
    from nano_qwen_b200.config import ModelConfig
    from nano_qwen_b200.models import Qwen3Model
    from nano_qwen_b200.training.optimizer import attach_param_store, build_optimizer
    torch.manual_seed(0)
    m = Qwen3Model(ModelConfig(**TINY))
    store = attach_param_store(m, torch.float32, torch.device("cpu"))
    opt = build_optimizer(m, lr=1e-3, fused=True, store=store)
    ids = torch.randint(0, 256, (2, 16))
    m(ids, labels=ids)["loss"].backward()
    ref = torch.sqrt(sum((p.grad.double() ** 2).sum() for p in m.parameters())).item()
    n = opt.clip_grad_norm_(1e-3)
    assert abs(float(n) - ref) < 1e-4 * ref
    assert abs(float(opt.clip_scale) - 1e-3 / (ref + 1e-6)) < 1e-6


@pytest.mark.skipif(not HAS_REF, reason="reference copy not present")
@pytest.mark.parametrize("kind", ["cosine", "wsd"])
def test_scheduler_matches_reference(kind):
    if REF not in sys.path:
        sys.path.append(REF)
    from training.scheduler import build_scheduler as ref_build
    from nano_qwen_b200.training.scheduler import build_scheduler
    p1 = [torch.nn.Parameter(torch.zeros(1))]
    p2 = [torch.nn.Parameter(torch.zeros(1))]
    o1 = torch.optim.SGD(p1, lr=1.0)
    o2 = torch.optim.SGD(p2, lr=1.0)
    kw = dict(warmup_steps=10, total_steps=100)
    if kind == "wsd":
        kw["stable_steps"] = 60
    s1 = ref_build(o1, scheduler_type=kind, **kw)
    s2 = build_scheduler(o2, scheduler_type=kind, **kw)
    for _ in range(100):
        assert math.isclose(s1.get_last_lr()[0], s2.get_last_lr()[0], rel_tol=1e-6, abs_tol=1e-9)
        o1.step(); o2.step(); s1.step(); s2.step()


# ------------------------------------------------------------------ checkpoint
def test_checkpoint_roundtrip_plain_and_dcp(tmp_path):
    from nano_qwen_b200.config import ModelConfig
    from nano_qwen_b200.models import Qwen3Model
    from nano_qwen_b200.training.checkpoint import CheckpointManager
    from nano_qwen_b200.training.engine import TrainEngine
    torch.manual_seed(0)
    cfg = ModelConfig(**TINY)
    tc = {"optimizer": {"lr": 1e-2}, "scheduler": {"warmup_steps": 0, "total_steps": 10}}
    eng = TrainEngine(Qwen3Model(cfg), tc, torch.device("cpu"))
    ids = torch.randint(0, 256, (2, 16))
    eng.train_step([{"input_ids": ids, "labels": ids}])
    mgr = CheckpointManager(save_dir=str(tmp_path), save_interval=1, async_save=False)
    model, opt, sch = eng.state_for_save()
    mgr.save(1, model, opt, sch, extra_state={"step": 1})
    path = mgr.latest()
    assert path is not None and os.path.exists(os.path.join(path, "meta.json"))
    eng2 = TrainEngine(Qwen3Model(cfg), tc, torch.device("cpu"))
    extra = mgr.load(eng2.model, eng2.optimizer, eng2.scheduler, path)
    assert int(extra.get("step", 0)) == 1
    for (n, p), (_, q) in zip(eng.model.named_parameters(), eng2.model.named_parameters()):
        assert torch.equal(p, q), n
    # the next step is identical after the reload
    o1 = eng.train_step([{"input_ids": ids, "labels": ids}])
    o2 = eng2.train_step([{"input_ids": ids, "labels": ids}])
    assert torch.allclose(o1["loss"], o2["loss"])
    for (n, p), (_, q) in zip(eng.model.named_parameters(), eng2.model.named_parameters()):
        assert torch.allclose(p, q, atol=1e-7), n
    out = str(tmp_path / "checkpoint.pt")
    mgr.export_plain(out, eng.model, step=2)
    from nano_qwen_b200.cli import load_model_for_eval
    import yaml
    yp = tmp_path / "m.yaml"
    yp.write_text(yaml.safe_dump(TINY))
    m3 = load_model_for_eval(str(yp), out)
    for (n, p), (_, q) in zip(eng.model.named_parameters(), m3.named_parameters()):
        assert torch.equal(p.detach(), q.detach()), n


def test_document_mask_and_padding_key_ranges():
    """Packed documents attend within themselves (the logits of each document
    equal its logits alone), and a left-padded row's real tokens ignore the
    padding; key ranges come from document ids or a one-run padding mask."""
    from nano_qwen_b200.config import ModelConfig
    from nano_qwen_b200.models import Qwen3Model
    from nano_qwen_b200.ops import KeyRange
    torch.manual_seed(2)
    m = Qwen3Model(ModelConfig(**dict(TINY, tie_word_embeddings=False))).eval()
    a = torch.randint(0, 256, (1, 11))
    b = torch.randint(0, 256, (1, 9))
    packed = torch.cat([a, b], 1)
    doc = torch.tensor([[0] * 11 + [1] * 9])
    pos = torch.cat([torch.arange(11), torch.arange(9)]).view(1, -1)
    with torch.no_grad():
        lp = m(packed, position_ids=pos, document_ids=doc)["logits"]
        assert torch.allclose(lp[:, :11], m(a)["logits"], atol=1e-5)
        assert torch.allclose(lp[:, 11:], m(b)["logits"], atol=1e-5)
        # left padding: 4 pad tokens, positions of the real tokens start at 0
        mask = torch.tensor([[0] * 4 + [1] * 9])
        padded = torch.cat([torch.zeros(1, 4, dtype=torch.long), b], 1)
        pos2 = torch.cat([torch.zeros(4, dtype=torch.long), torch.arange(9)]).view(1, -1)
        lpad = m(padded, position_ids=pos2, attention_mask=mask)["logits"]
        assert torch.allclose(lpad[:, 4:], m(b)["logits"], atol=1e-5)
    kr = KeyRange.from_segments(torch.tensor([[0, 0, 0, 1, 1, 2, 2, 2]]))
    assert kr.kv_lo.tolist() == [[0, 0, 0, 3, 3, 5, 5, 5]]
    assert kr.q_hi.tolist() == [[3, 3, 3, 5, 5, 8, 8, 8]]
    assert KeyRange.from_padding_mask(torch.tensor([[1, 1, 0, 1]])) is None  # two runs of real tokens
    assert KeyRange.from_padding_mask(torch.tensor([[0, 1, 1, 0]])).kv_lo.tolist() == [[0, 1, 1, 3]]


@pytest.mark.skipif(not HAS_REF, reason="reference copy not present")
@pytest.mark.parametrize("dcfg", [{"beta": 0.1}, {"beta": 0.5, "label_smoothing": 0.1},
                                  {"beta": 0.2, "reference_free": True}])
def test_dpo_loss_matches_reference(dcfg):
    """The DPO objective (mean per-token log-ratio scores, sigmoid loss,
    label smoothing, reference-free mode) against the reference trainer on
    the same weights and pairs: loss value and policy gradients."""
    RC, RM = _ref_import()
    from training.dpo import DPOTrainer as RefDPO

    from nano_qwen_b200.config import ModelConfig
    from nano_qwen_b200.models import Qwen3Model
    from nano_qwen_b200.training.dpo import DPOTrainer
    torch.manual_seed(0)
    ref_policy, ref_ref = RM(RC(**TINY)), RM(RC(**TINY))
    pol, refm = Qwen3Model(ModelConfig(**TINY)), Qwen3Model(ModelConfig(**TINY))
    pol.load_state_dict(ref_policy.state_dict())
    refm.load_state_dict(ref_ref.state_dict())
    cfg = {"dpo": dcfg, "optimizer": {"lr": 1e-3}}
    a = RefDPO(ref_policy, ref_ref, cfg, torch.device("cpu"))
    b = DPOTrainer(pol, refm, cfg, torch.device("cpu"))
    g = torch.Generator().manual_seed(1)
    c_ids, r_ids = (torch.randint(0, TINY["vocab_size"], (3, 20), generator=g) for _ in range(2))
    # (the reference gathers log-probabilities before masking, so it cannot
    # take -100 labels; ours masks prompt tokens, checked below)
    c_lab, r_lab = c_ids.clone(), r_ids.clone()
    la, _ = a.dpo_loss(c_ids, r_ids, c_lab, r_lab)
    lb, _ = b.dpo_loss(c_ids, r_ids, c_lab, r_lab)
    assert torch.allclose(la, lb, atol=1e-5, rtol=1e-5), (float(la), float(lb))
    la.backward()
    lb.backward()
    rp = dict(ref_policy.named_parameters())
    for n, p in b.policy.named_parameters():
        assert torch.allclose(p.grad, rp[n].grad, atol=1e-5, rtol=1e-3), n
    c_lab[:, :6] = -100          # prompt tokens carry no score
    r_lab[:, :6] = -100
    lm, _ = b.dpo_loss(c_ids, r_ids, c_lab, r_lab)
    assert torch.isfinite(lm)


@pytest.mark.skipif(not HAS_REF, reason="reference copy not present")
def test_evaluator_and_reward_model_match_reference():
    """Perplexity, multiple-choice scoring and the reward model's
    Bradley-Terry loss against the reference's on the same weights."""
    RC, RM = _ref_import()
    from eval.evaluate import Evaluator as RefEval
    from training.reward_model import RewardModel as RefRM

    from nano_qwen_b200.config import ModelConfig
    from nano_qwen_b200.data.tokenizer import Tokenizer
    from nano_qwen_b200.eval.evaluate import Evaluator
    from nano_qwen_b200.models import Qwen3Model
    from nano_qwen_b200.training.reward_model import RewardModel
    torch.manual_seed(0)
    cfg = dict(TINY, vocab_size=300)
    ref = RM(RC(**cfg)).eval()
    ours = Qwen3Model(ModelConfig(**cfg)).eval()
    ours.load_state_dict(ref.state_dict())
    tok = Tokenizer(backend="bytes")
    g = torch.Generator().manual_seed(2)
    batches = []
    for _ in range(3):
        ids = torch.randint(0, 256, (2, 20), generator=g)
        lab = ids.clone()
        lab[:, :3] = -100
        batches.append({"input_ids": ids, "labels": lab})
    dev = torch.device("cpu")
    with torch.no_grad():
        pa = RefEval(ref, tok, dev).compute_perplexity(batches)
        pb = Evaluator(ours, tok, dev).compute_perplexity(batches)
    assert abs(pa - pb) < 1e-3 * pa, (pa, pb)
    qs = [{"prompt": f"question {i}?", "choices": ["alpha", "beta", "gamma", "delta"], "answer": i % 4}
          for i in range(4)]
    ra = RefEval(ref, tok, dev).eval_multiple_choice(qs)
    rb = Evaluator(ours, tok, dev).eval_multiple_choice(qs)
    assert ra["correct"] == rb["correct"] and ra["total"] == rb["total"], (ra, rb)
    rr = RefRM(RC(**cfg))
    rm = RewardModel(ModelConfig(**cfg))
    missing, unexpected = rm.load_state_dict(rr.state_dict(), strict=False)
    assert not unexpected and all("lm_head" in k for k in missing), (missing, unexpected)
    c, r = torch.randint(0, 256, (3, 16), generator=g), torch.randint(0, 256, (3, 16), generator=g)
    # (the reference's attention cannot take a [B, S] padding mask, so the
    # comparison pools the last position of unpadded rows)
    la = rr.compute_preference_loss(c, r)["loss"]
    lb = rm.compute_preference_loss(c, r)["loss"]
    assert torch.allclose(la, lb, atol=1e-5, rtol=1e-5), (float(la), float(lb))
    # ours takes right-padded rows: the last real token is pooled
    mask = torch.ones(3, 16, dtype=torch.long)
    mask[0, 12:] = 0
    padded = rm.compute_preference_loss(c, r, mask, mask)
    trimmed = rm(c[:1, :12])
    assert torch.allclose(rm(c, mask)[0], trimmed[0], atol=1e-5), "pooling of a padded row"
    assert torch.isfinite(padded["loss"])


@pytest.mark.skipif(not HAS_REF, reason="reference copy not present")
def test_grpo_reward_and_advantages_match_reference():
    """The verifiable math reward (\\boxed{}, '####', last number) and the
    group-normalised advantages against the reference's."""
    _ref_import()
    from training.grpo import GRPO as RefGRPO, _math_reward_fn as ref_reward

    from nano_qwen_b200.training.grpo import GRPO, _math_reward_fn
    responses = ["so the answer is \\\\boxed{42}", "#### 41", "I think 42.0", "no idea", "x = -3",
                 "\\\\boxed{forty-two}", "12 then 42", ""]
    for gt in ("42", "#### 42", "\\\\boxed{-3}", "forty-two", None):
        assert _math_reward_fn(responses, gt) == ref_reward(responses, gt), gt
    rewards = torch.tensor([1.0, 0.0, 1.0, 0.0, 0.0, 1.0])
    ref_adv = RefGRPO.compute_advantages(None, rewards)   # a method that uses no state
    assert torch.allclose(GRPO.compute_advantages(rewards), ref_adv, atol=1e-6)


@pytest.mark.skipif(not HAS_REF, reason="reference copy not present")
def test_chat_format_matches_reference():
    """The SFT chat template (thinking, empty thinking, plain) is the
    reference's text exactly: checkpoints trained on either format the same
    prompts."""
    _ref_import()
    from training.sft import format_conversation as ref_fmt

    from nano_qwen_b200.training.sft import format_conversation
    for reasoning in ("step 1\nstep 2", None):
        for think in (True, False):
            args = ("be brief", "What is 2+2?", "4", reasoning, think)
            assert format_conversation(*args) == ref_fmt(*args)
