"""CPU runs of the data pipeline, every training phase through the CLI, and
evaluation (tiny model, synthetic / fallback data, temporary directories)."""

import json
import os

import pytest
import torch
import yaml

MODEL = dict(hidden_size=64, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
             head_dim=16, intermediate_size=128, vocab_size=300, max_position_embeddings=256,
             tie_word_embeddings=True)
TRAIN = {
    "optimizer": {"lr": 1e-3, "weight_decay": 0.1, "grad_clip": 1.0},
    "scheduler": {"type": "cosine", "warmup_steps": 1, "total_steps": 4},
    "batch": {"micro_batch_size": 2, "gradient_accumulation_steps": 2, "max_seq_len": 32},
    "checkpoint": {"save_interval": 2, "save_dir": "ck", "async_save": False},
    "logging": {"log_interval": 1, "tensorboard_enabled": False, "wandb_enabled": False},
    "data": {"train_data": "nodata", "num_workers": 0},
    "grpo": {"group_size": 2, "max_gen_len": 8},
    "dpo": {"beta": 0.1},
}


@pytest.fixture
def cfgs(tmp_path, monkeypatch):
    monkeypatch.chdir(tmp_path)
    (tmp_path / "m.yaml").write_text(yaml.safe_dump(MODEL))
    (tmp_path / "t.yaml").write_text(yaml.safe_dump(TRAIN))
    return str(tmp_path / "m.yaml"), str(tmp_path / "t.yaml")


# ------------------------------------------------------------------ data
def test_packed_dataset_and_sampler_resume():
    from nano_qwen_b200.data.dataset import PackedTextDataset
    from nano_qwen_b200.data.sampler import DistributedSampler
    ds = PackedTextDataset(data_dir="does-not-exist", max_seq_len=16, vocab_size=100)
    item = ds[0]
    assert item["input_ids"].shape == (16,) and int(item["input_ids"].max()) < 100
    s = DistributedSampler(ds, num_replicas=2, rank=1, shuffle=True, seed=3)
    order = list(iter(s))
    s2 = DistributedSampler(ds, num_replicas=2, rank=1, shuffle=True, seed=3)
    s2.set_start_index(5)
    assert list(iter(s2)) == order[5:]
    other = list(iter(DistributedSampler(ds, num_replicas=2, rank=0, shuffle=True, seed=3)))
    assert not set(order) & set(other)


def test_packed_dataset_reads_token_files(tmp_path):
    import numpy as np
    from nano_qwen_b200.data.dataset import PackedTextDataset
    toks = np.arange(1000, dtype=np.uint16) % 77
    toks.tofile(tmp_path / "shard0.bin")
    ds = PackedTextDataset(data_dir=str(tmp_path), max_seq_len=10, vocab_size=77, dtype=np.uint16)
    assert len(ds) > 0
    a = ds[0]["input_ids"]
    assert a.tolist() == (np.arange(10) % 77).tolist()
    assert ds._native is not None  # the C++ reader is built in-tree
    (np.arange(5, dtype=np.uint16) + 3).tofile(tmp_path / "shard1.bin")
    ds2 = PackedTextDataset(data_dir=str(tmp_path), max_seq_len=10, vocab_size=77,
                            dtype=np.uint16, eos_id=0)
    native = ds2._window(995, 12)
    ds2._native = None
    assert native.tolist() == ds2._window(995, 12).tolist()  # spans both shards + padding


def test_tokenizer_roundtrip_bytes():
    from nano_qwen_b200.data.tokenizer import Tokenizer
    tok = Tokenizer(backend="bytes")
    s = "hello, world <think>x</think>"
    assert tok.decode(tok.encode(s, allowed_special="all")) == s


def test_sft_masks_prompt_tokens():
    from nano_qwen_b200.data.tokenizer import Tokenizer
    from nano_qwen_b200.training.sft import SFTDataset
    tok = Tokenizer(backend="bytes")
    ds = SFTDataset([{"system": "sys", "conversations": [{"user": "what?", "assistant": "this."}]}],
                    tok, max_seq_len=160)
    it = ds[0]
    ids, labels = it["input_ids"], it["labels"]
    supervised = labels != -100
    assert supervised.any() and (~supervised).any()
    text = tok.decode(ids[supervised].tolist())
    assert "this." in text and "what?" not in text


# ------------------------------------------------------------------ CLI
def test_cli_pretrain_and_resume(cfgs):
    from nano_qwen_b200.cli import main
    m, t = cfgs
    assert main(["pretrain", "--model-config", m, "--training-config", t, "--max-steps", "2"]) == 0
    assert os.path.isdir("ck/step_00000002")
    assert main(["pretrain", "--model-config", m, "--training-config", t, "--max-steps", "4",
                 "--resume", "ck/step_00000002"]) == 0
    assert os.path.isdir("ck/step_00000004")


@pytest.mark.parametrize("cmd", ["sft", "dpo", "grpo"])
def test_cli_post_training_phases(cfgs, cmd):
    """Each phase runs, checkpoints every ``save_interval`` steps, and resumes
    from the newest checkpoint when the YAML says ``resume_from: latest``."""
    from nano_qwen_b200.cli import main
    m, t = cfgs
    assert main([cmd, "--model-config", m, "--training-config", t, "--max-steps", "2",
                 "--max-samples", "8"]) == 0
    assert os.path.isdir("ck/step_00000002")
    cfg = yaml.safe_load(open(t))
    cfg["checkpoint"]["resume_from"] = "latest"
    with open(t, "w") as f:
        yaml.safe_dump(cfg, f)
    assert main([cmd, "--model-config", m, "--training-config", t, "--max-steps", "4",
                 "--max-samples", "8"]) == 0
    assert os.path.isdir("ck/step_00000004")
    meta = json.load(open("ck/step_00000004/meta.json"))
    assert meta["step"] == 4


def test_grpo_reward_types_combine():
    """``grpo.reward_types`` / ``reward_weights`` select and weight reward
    sources; a model reward without a checkpoint is skipped."""
    from nano_qwen_b200.training.grpo import build_reward_fn
    fn = build_reward_fn({"grpo": {"reward_types": ["verifiable", "model"],
                                   "reward_weights": [2.0, 1.0]}})
    assert [k for k, _, _ in fn.fns] == ["verifiable"]
    fn.set_prompt("What is 6 * 7?")
    assert fn(["It is 42.", "\\boxed{41}"], "42") == [2.0, 0.0]
    with pytest.raises(ValueError):
        build_reward_fn({"grpo": {"reward_types": ["nonsense"]}})


def test_cli_eval_multiple_choice(cfgs, tmp_path):
    from nano_qwen_b200.cli import main
    from nano_qwen_b200.config import ModelConfig
    from nano_qwen_b200.models import Qwen3Model
    m, _ = cfgs
    torch.save({"model": Qwen3Model(ModelConfig(**MODEL)).state_dict()}, tmp_path / "checkpoint.pt")
    os.makedirs("benchmarks", exist_ok=True)
    with open("benchmarks/toy.jsonl", "w") as f:
        for i in range(3):
            f.write(json.dumps({"prompt": f"q{i}", "choices": ["a", "b"], "answer": 0}) + "\n")
    assert main(["eval", "--model-config", m, "--checkpoint", str(tmp_path / "checkpoint.pt"),
                 "--benchmarks", "toy", "--output", "res.json"]) == 0
    res = json.load(open("res.json"))
    assert res["toy"]["total"] == 3


def test_generation_greedy_is_deterministic():
    from nano_qwen_b200.config import ModelConfig
    from nano_qwen_b200.data.tokenizer import Tokenizer
    from nano_qwen_b200.eval.generate import TextGenerator
    from nano_qwen_b200.models import Qwen3Model
    torch.manual_seed(0)
    g = TextGenerator(Qwen3Model(ModelConfig(**MODEL)), Tokenizer(backend="bytes"))
    a = g.generate("abc", max_new_tokens=6, temperature=0.0)
    b = g.generate("abc", max_new_tokens=6, temperature=0.0)
    assert a == b


def test_tracing_nvtx_and_step_profiler(tmp_path):
    """NVTX ranges are inert without a GPU and when off; the step profiler
    writes a trace and a kernel table after its window."""
    import torch
    from nano_qwen_b200.utils.tracing import StepProfiler, enable_nvtx, nvtx_range
    enable_nvtx(True)
    with nvtx_range("x"):
        pass
    enable_nvtx(False)
    prof = StepProfiler(str(tmp_path), wait=1, warmup=1, active=2)
    for i in range(5):
        with prof.step(i):
            torch.randn(64, 64) @ torch.randn(64, 64)
    assert prof.done
    assert (tmp_path / "trace_rank0.json").exists() and (tmp_path / "kernels_rank0.txt").exists()


def test_replay_step_is_bitwise_on_cpu():
    """The replay check restores the full state: on the CPU path a step is
    bit-identical run to run."""
    import torch
    from nano_qwen_b200.config import ModelConfig
    from nano_qwen_b200.models import Qwen3Model
    from nano_qwen_b200.training.engine import TrainEngine
    from nano_qwen_b200.utils.replay import replay_step
    torch.manual_seed(0)
    cfg = ModelConfig(hidden_size=64, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                      head_dim=16, intermediate_size=128, vocab_size=256, max_position_embeddings=64)
    eng = TrainEngine(Qwen3Model(cfg), {"optimizer": {"lr": 1e-2}, "scheduler": {"warmup_steps": 0}},
                      torch.device("cpu"))
    ids = torch.randint(0, 256, (2, 16))
    eng.train_step([{"input_ids": ids, "labels": ids}])
    r = replay_step(eng, [{"input_ids": ids, "labels": ids}])
    assert r["loss_equal"] and not r["differs"], r


def test_cli_nproc_relaunch_command():
    """``--nproc N`` turns the command into a one-process-per-GPU launch on
    this node (the reference's torchrun shell wrappers)."""
    import os
    from nano_qwen_b200.cli import relaunch_argv
    assert relaunch_argv(["pretrain", "--model-config", "m.yaml"]) is None
    assert relaunch_argv(["--nproc", "1", "pretrain", "--model-config", "m.yaml"]) is None
    cmd = relaunch_argv(["--nproc", "4", "sft", "--model-config", "m.yaml", "--variant", "fusion"])
    assert cmd[1:4] == ["-m", "torch.distributed.run", "--standalone"]
    assert "--nproc-per-node=4" in cmd and "127.0.0.1" in cmd
    assert cmd[-5:] == ["sft", "--model-config", "m.yaml", "--variant", "fusion"]
    os.environ["LOCAL_RANK"] = "0"
    try:
        assert relaunch_argv(["--nproc", "4", "pretrain"]) is None
    finally:
        del os.environ["LOCAL_RANK"]


@pytest.mark.parametrize("cmd", ["pretrain", "grpo"])
def test_cli_fully_sharded_runs_and_resumes(tmp_path, monkeypatch, cmd):
    """``distributed.shard_params`` (fully sharded parameters) through the
    CLI: pretraining with checkpoint + resume, and GRPO, whose rollouts run
    the sharded model's generation."""
    from nano_qwen_b200.cli import main
    monkeypatch.chdir(tmp_path)
    t = dict(TRAIN, distributed={"shard_params": True})
    (tmp_path / "m.yaml").write_text(yaml.safe_dump(MODEL))
    (tmp_path / "t.yaml").write_text(yaml.safe_dump(t))
    args = ["--model-config", "m.yaml", "--training-config", "t.yaml"]
    assert main([cmd] + args + ["--max-steps", "2"]) == 0
    if cmd == "pretrain":
        assert os.path.isdir("ck/step_00000002")
        assert main([cmd] + args + ["--max-steps", "4", "--resume", "ck/step_00000002"]) == 0
        assert os.path.isdir("ck/step_00000004")


def test_fully_sharded_single_process_matches_flat_store():
    """One rank: the fully sharded store (units gathered and released around
    every block, gradients reduced per block) trains exactly like the flat
    store."""
    from nano_qwen_b200.config import ModelConfig
    from nano_qwen_b200.models import Qwen3Model
    from nano_qwen_b200.training.engine import TrainEngine
    cfg = ModelConfig(**dict(MODEL, gradient_checkpointing=True))
    tc = {"optimizer": {"lr": 1e-2, "grad_clip": 1.0},
          "scheduler": {"warmup_steps": 0, "total_steps": 10}}
    engines = []
    for shard in (False, True):
        torch.manual_seed(0)
        engines.append(TrainEngine(Qwen3Model(cfg), dict(tc, distributed={"shard_params": shard}),
                                   torch.device("cpu")))
    plain, fs = engines
    assert fs.store.mode == "fsdp"
    g = torch.Generator().manual_seed(3)
    for _ in range(3):
        ids = torch.randint(0, cfg.vocab_size, (4, 32), generator=g)
        mbs = [{"input_ids": ids[i:i + 2], "labels": ids[i:i + 2]} for i in (0, 2)]
        a, b = plain.train_step(mbs), fs.train_step(mbs)
        assert torch.allclose(a["loss"], b["loss"], rtol=1e-6, atol=1e-6)
        assert torch.allclose(a["grad_norm"], b["grad_norm"], rtol=1e-5)
    fs.state_for_save()
    for (n, p), (_, q) in zip(plain.model.named_parameters(), fs.model.named_parameters()):
        assert torch.allclose(p, q, rtol=1e-5, atol=1e-6), n
    fs.optimizer.release_full_state()
    mem = fs.store.memory_bytes()
    assert mem["shards"] > 0 and mem["largest_block_unit"] > 0


def test_fully_sharded_memory_plan():
    """The memory plan of the fully sharded layout (a meta-device model, no
    allocation): the per-rank state falls with the world size (18 B per
    element over the ranks, up to unit padding), below ZeRO-2's."""
    from nano_qwen_b200.config import ModelConfig
    from nano_qwen_b200.models import Qwen3Model
    from nano_qwen_b200.parallel.fsdp import memory_plan
    with torch.device("meta"):
        m = Qwen3Model(ModelConfig(**dict(MODEL, hidden_size=256, intermediate_size=512,
                                          vocab_size=4096, num_hidden_layers=4)))
    one, eight = memory_plan(m, 1), memory_plan(m, 8)
    n = one["params"]
    assert abs(one["fsdp_state"] - 18 * n) < 0.05 * 18 * n
    assert eight["fsdp_state"] < one["fsdp_state"] / 7
    assert eight["fsdp_total"] < eight["zero2_state"]


def test_expert_parallel_zero2_memory_plan():
    """ZeRO-2 under expert parallelism: one rank holds 1/ep of the experts;
    sharding their moments over the world / ep ranks holding the same
    experts (and the dense moments over the world) against keeping every
    moment of the rank's parameters, by the element counts."""
    from nano_qwen_b200.config import ModelConfig
    from nano_qwen_b200.models import Qwen3Model
    from nano_qwen_b200.parallel.fsdp import memory_plan
    with torch.device("meta"):
        m = Qwen3Model(ModelConfig(**dict(MODEL, hidden_size=256, intermediate_size=512,
                                          vocab_size=4096, num_hidden_layers=4, num_experts=8,
                                          num_experts_per_tok=2, moe_intermediate_size=128)))
    n = sum(p.numel() for p in m.parameters())
    x = sum(p.numel() for k, p in m.named_parameters() if ".experts." in k)
    plan = memory_plan(m, 8, ep=2)
    local = (n - x) + x / 2
    assert abs(plan["zero2_ep_replicated_state"] - local * 18) < 1
    assert abs(plan["zero2_ep_state"] - (local * 10 + (n - x) * 8 / 8 + x / 2 * 8 / 4)) < 1
    assert plan["zero2_ep_state"] < plan["zero2_ep_replicated_state"]
    assert "zero2_ep_state" not in memory_plan(m, 8)


@pytest.mark.parametrize("moe", [False, True])
def test_cached_generation_paths_match_full_forward_on_cpu(moe):
    """The three inference paths agree with one full forward (fp32, CPU):
    the model with a growing KV cache, and the static-cache decode step the
    generator uses (prefill, then one token at a time at the right
    positions), batch of two."""
    from nano_qwen_b200.config import ModelConfig
    from nano_qwen_b200.eval.generate import DecodeState, decode_step, prefill
    from nano_qwen_b200.models import KVCache, Qwen3Model
    torch.manual_seed(0)
    extra = dict(num_experts=4, num_experts_per_tok=2, moe_intermediate_size=32) if moe else {}
    cfg = ModelConfig(**dict(MODEL, **extra))
    m = Qwen3Model(cfg).eval()
    ids = torch.randint(0, cfg.vocab_size, (2, 24))
    with torch.no_grad():
        full = m(ids, return_logits=True)["logits"]
        caches = [KVCache() for _ in range(cfg.num_hidden_layers)]
        steps = [m(ids[:, :16], kv_caches=caches, return_logits=True)["logits"][:, -1]]
        for t in range(16, 23):
            steps.append(m(ids[:, t:t + 1], kv_caches=caches, return_logits=True)["logits"][:, -1])
        torch.testing.assert_close(torch.stack(steps, 1), full[:, 15:23], rtol=1e-4, atol=1e-4)
        st = DecodeState(m, 2, 32, torch.device("cpu"), torch.float32)
        got = [prefill(m, st, ids[:, :16])]
        for t in range(16, 23):
            st.ids.copy_(ids[:, t:t + 1])
            got.append(decode_step(m, st))
        torch.testing.assert_close(torch.stack(got, 1), full[:, 15:23].float(), rtol=1e-4, atol=1e-4)
