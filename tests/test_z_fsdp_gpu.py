"""Fully sharded parameters on the GPU (one rank): the store gathers each
block's bf16 weights into a buffer that is released after use, the GEMMs read
and write views of those buffers, and training must match the flat store
step for step.  (The multi-rank schedule is covered with Gloo ranks on the
CPU.)"""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _cfg(**kw):
    from nano_qwen_b200.config import ModelConfig
    base = dict(hidden_size=256, num_hidden_layers=3, num_attention_heads=4, num_key_value_heads=2,
                head_dim=64, intermediate_size=512, vocab_size=4096, max_position_embeddings=512,
                tie_word_embeddings=True, rope_theta=1e4)
    base.update(kw)
    return ModelConfig(**base)


@pytest.mark.parametrize("ckpt", [False, True])
def test_fully_sharded_store_matches_flat_store(ckpt):
    from nano_qwen_b200.models import Qwen3Model
    from nano_qwen_b200.parallel.fsdp import _FREE
    from nano_qwen_b200.training.engine import TrainEngine
    dev = torch.device("cuda", 0)
    cfg = _cfg(gradient_checkpointing=ckpt)
    tc = {"optimizer": {"lr": 1e-3, "grad_clip": 1.0},
          "scheduler": {"warmup_steps": 0, "total_steps": 10}}
    engines = []
    for shard in (False, True):
        torch.manual_seed(0)
        engines.append(TrainEngine(Qwen3Model(cfg), dict(tc, distributed={"shard_params": shard}),
                                   dev))
    plain, fs = engines
    st = fs.store
    assert st.mode == "fsdp" and st.compute.dtype == torch.bfloat16
    g = torch.Generator().manual_seed(3)
    for _ in range(3):
        ids = torch.randint(0, cfg.vocab_size, (4, 256), generator=g).to(dev)
        mbs = [{"input_ids": ids[i:i + 2], "labels": ids[i:i + 2]} for i in (0, 2)]
        a, b = plain.train_step(mbs), fs.train_step(mbs)
        torch.testing.assert_close(b["loss"], a["loss"], rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(b["grad_norm"], a["grad_norm"], rtol=1e-4, atol=1e-6)
        # block weights and every full gradient buffer are released between steps
        assert all(u.state == _FREE for u in st.block_units[:-1])
        assert not any(u.grad_live for u in st.units)
    torch.cuda.synchronize()
    fs.state_for_save()
    for (n, p), (_, q) in zip(plain.model.named_parameters(), fs.model.named_parameters()):
        torch.testing.assert_close(q, p, rtol=1e-4, atol=1e-5, msg=n)
    fs.optimizer.release_full_state()
