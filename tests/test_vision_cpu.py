"""CPU tests of the vision-language stack: the reference's Qwen3VLModel and
vision modules (imported read-only from ``baseline/_ref``) as oracles, an
fp32 restatement of multimodal RoPE (which the reference never wires into
attention), and the image preprocessing / multimodal dataset."""

import math
import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")
HAS_REF = os.path.isdir(os.path.join(REF, "model"))
needs_ref = pytest.mark.skipif(not HAS_REF, reason="reference copy not present")

VL = dict(hidden_size=64, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
          head_dim=16, intermediate_size=128, vocab_size=256, max_position_embeddings=128,
          tie_word_embeddings=True, vision_enabled=True, vision_hidden_size=48,
          vision_num_hidden_layers=3, vision_num_attention_heads=4, vision_intermediate_size=96,
          vision_patch_size=4, vision_image_size=32, vision_num_channels=3,
          vision_deepstack_layers=[0, 1], vision_merger_spatial_factor=2)


def _ref(mod, name):
    if REF not in sys.path:
        sys.path.append(REF)
    return getattr(__import__(mod, fromlist=[name]), name)


def _batch(seed=0, B=2, S=40, n_img_tok=16):
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, VL["vocab_size"], (B, S), generator=g)
    mask = torch.zeros(B, S, dtype=torch.bool)
    mask[0, 4:4 + n_img_tok] = True
    mask[1, 10:10 + n_img_tok] = True
    px = torch.randn(B, 3, VL["vision_image_size"], VL["vision_image_size"], generator=g)
    return ids, mask, px


def _pair():
    RC = _ref("model.config", "ModelConfig")
    RVL = _ref("model.multimodal", "Qwen3VLModel")
    from nano_qwen_b200.config import ModelConfig
    from nano_qwen_b200.models.multimodal import Qwen3VLModel
    torch.manual_seed(0)
    ref = RVL(RC(**VL))
    ours = Qwen3VLModel(ModelConfig(**VL))
    ours.load_state_dict(ref.state_dict())
    return ref, ours


def _rel(a, b):
    a, b = a.detach().double(), b.detach().double()
    return ((a - b).norm() / (b.norm() + 1e-30)).item()


@needs_ref
def test_vl_model_matches_reference_loss_and_grads():
    """With MRoPE off (the reference never applies it), loss and every
    gradient equal the reference's on images + text."""
    ref, ours = _pair()
    ours.use_mrope = False
    ids, mask, px = _batch()
    a = ref(ids, pixel_values=px, image_token_mask=mask, labels=ids)
    b = ours(ids, pixel_values=px, image_token_mask=mask, labels=ids)
    assert torch.allclose(a["loss"], b["loss"], atol=1e-5, rtol=1e-5), (a["loss"], b["loss"])
    a["loss"].backward()
    b["loss"].backward()
    rg = dict(ref.named_parameters())
    for n, p in ours.named_parameters():
        if rg[n].grad is None:
            assert p.grad is None or p.grad.abs().max() == 0, n
            continue
        assert _rel(p.grad, rg[n].grad) < 1e-4, (n, _rel(p.grad, rg[n].grad))


@needs_ref
@pytest.mark.parametrize("part", ["vit", "deepstack", "merger", "patch"])
def test_vision_modules_match_reference(part):
    from nano_qwen_b200.config import ModelConfig
    cfg = ModelConfig(**VL)
    RC = _ref("model.config", "ModelConfig")
    rcfg = RC(**VL)
    torch.manual_seed(1)
    g = torch.Generator().manual_seed(2)
    if part == "vit":
        ours = __import__("nano_qwen_b200.models.vision.vit", fromlist=["x"]).VisionTransformer(cfg)
        ref = _ref("model.vision.vit", "VisionTransformer")(rcfg)
        # a second resolution exercises the bilinear position-embedding resize
        for size in (32, 48):
            x = torch.randn(2, 3, size, size, generator=g)
            ref.load_state_dict(ours.state_dict())
            a, b = ref(x), ours(x)
            assert _rel(b["last_hidden_state"], a["last_hidden_state"]) < 1e-5
            assert len(a["intermediate_states"]) == len(b["intermediate_states"]) == 2
            for u, v in zip(b["intermediate_states"], a["intermediate_states"]):
                assert _rel(u, v) < 1e-5
        return
    if part == "deepstack":
        ours = __import__("nano_qwen_b200.models.vision.deepstack", fromlist=["x"]).DeepStack(48, 64, 3)
        ref = _ref("model.vision.deepstack", "DeepStack")(48, 64, 3)
        ref.load_state_dict(ours.state_dict())
        with torch.no_grad():
            ours.fusion_weights.copy_(torch.tensor([0.3, -0.2, 1.1]))
            ref.fusion_weights.copy_(ours.fusion_weights)
        st = [torch.randn(2, 64, 48, generator=g) for _ in range(3)]
        assert _rel(ours(st[:2], st[2]), ref(st[:2], st[2])) < 1e-5
        assert _rel(ours(st[:1], st[2]), ref(st[:1], st[2])) < 1e-5  # level-count fallback
        return
    if part == "merger":
        ours = __import__("nano_qwen_b200.models.vision.merger", fromlist=["x"]).VisionMerger(64, 64, 2)
        ref = _ref("model.vision.merger", "VisionMerger")(64, 64, 2)
        ref.load_state_dict(ours.state_dict())
        x = torch.randn(2, 64, 64, generator=g)
        assert _rel(ours(x, 8, 8), ref(x, 8, 8)) < 1e-5
        return
    ours = __import__("nano_qwen_b200.models.vision.patch_embed", fromlist=["x"]).PatchEmbedding(cfg)
    ref = _ref("model.vision.patch_embed", "PatchEmbedding")(rcfg)
    ref.load_state_dict(ours.state_dict())
    x = torch.randn(2, 3, 32, 32, generator=g)
    assert _rel(ours(x), ref(x)) < 1e-5


def _mrope_positions_oracle(text_pos, grids, mask):
    """Restated: image tokens of a row, in order across the row's images, take
    (t, h, w) of the concatenated grids enumerated t-major, then h, then w;
    text tokens keep their 1-D position in all three components."""
    B, S = text_pos.shape
    coords = [(t, h, w) for (T, H, W) in grids for t in range(T) for h in range(H) for w in range(W)]
    out = [text_pos.clone() for _ in range(3)]
    for b in range(B):
        k = 0
        for s in range(S):
            if mask[b, s] and k < len(coords):
                for c in range(3):
                    out[c][b, s] = coords[k][c]
                k += 1
    return out


def test_mrope_positions_and_tables_match_fp64_statement():
    from nano_qwen_b200.models.vision.mrope import build_mrope_position_ids, mrope_tables
    B, S = 2, 40
    ids, mask, _ = _batch(B=B, S=S)
    text = torch.arange(S).unsqueeze(0).expand(B, S).clone() + torch.tensor([[0], [5]])
    grids = [[1, 4, 4]]
    got = build_mrope_position_ids(text, torch.tensor(grids), mask)
    want = _mrope_positions_oracle(text, grids, mask)
    for g_, w_ in zip(got, want):
        assert torch.equal(g_, w_)
    D, base = 48, 1e4
    for sections in (None, [6, 8, 10]):
        cos, sin = mrope_tables(D, base, got, sections)
        half = D // 2
        if sections is None:
            sec = D // 3
            sections_ = [sec // 2, sec // 2, half - 2 * (sec // 2)]
        else:
            sections_ = sections
        comp = [c for c, n in enumerate(sections_) for _ in range(n)]
        inv = [base ** (-(2.0 * i) / D) for i in range(half)]
        for t in (0, 5, 17, 50, 79):
            b, s = divmod(t, S)
            for i in range(half):
                ang = float(got[comp[i]][b, s]) * inv[i]
                assert abs(float(cos[t, i]) - math.cos(ang)) < 2e-5
                assert abs(float(sin[t, i]) - math.sin(ang)) < 2e-5


def test_mrope_with_text_positions_equals_plain_rope_in_the_model():
    """The per-token MRoPE tables feed the same fused RoPE path: with every
    component equal to the 1-D position the model output is that of plain
    RoPE; with image grids it differs (MRoPE is applied)."""
    from nano_qwen_b200.config import ModelConfig
    from nano_qwen_b200.models.multimodal import Qwen3VLModel
    from nano_qwen_b200.models.vision.mrope import mrope_tables
    torch.manual_seed(0)
    m = Qwen3VLModel(ModelConfig(**VL))
    ids, mask, px = _batch()
    B, S = ids.shape
    pos = torch.arange(S).unsqueeze(0).expand(B, S)
    lm = m.language_model
    with torch.no_grad():
        x0, _, _ = lm.hidden(ids, None, None, None)
        tables = mrope_tables(VL["head_dim"], lm.config.rope_theta, (pos, pos, pos))
        x1, _, _ = lm.hidden(ids, None, None, None, rope=tables)
        assert _rel(x1, x0) < 1e-6
        on = m(ids, pixel_values=px, image_token_mask=mask)["logits"]
        m.use_mrope = False
        off = m(ids, pixel_values=px, image_token_mask=mask)["logits"]
    assert _rel(on, off) > 1e-4


@needs_ref
def test_image_processor_and_dataset_match_reference():
    from PIL import Image
    from nano_qwen_b200.data.multimodal_dataset import ImageProcessor, MultimodalDataset
    RIP = _ref("data.multimodal_dataset", "ImageProcessor")
    RMD = _ref("data.multimodal_dataset", "MultimodalDataset")
    g = torch.Generator().manual_seed(3)
    imgs = [Image.fromarray((torch.rand(h, w, 3, generator=g) * 255).to(torch.uint8).numpy())
            for h, w in ((50, 70), (97, 40), (64, 64))]
    ours, ref = ImageProcessor(image_size=56, patch_size=14), RIP(image_size=56, patch_size=14)
    for im in imgs:
        a, b = ours(im), ref(im)
        assert a.shape == b.shape == (3, 56, 56)
        assert (a - b).abs().max() < 1e-4
    assert ours.num_merged_tokens == ref.num_merged_tokens == 4
    samples = [{"text": list(range(10, 40)), "images": imgs[:2], "image_positions": [3, 20]}]
    S = 48
    a = MultimodalDataset(samples, image_processor=ours, max_seq_len=S)[0]
    b = RMD(samples, image_processor=ref, max_seq_len=S)[0]
    assert torch.equal(a["input_ids"], b["input_ids"])
    assert torch.equal(a["image_token_mask"], b["image_token_mask"])
    assert torch.allclose(a["pixel_values"], b["pixel_values"], atol=1e-4)
    # labels aligned with input_ids (the model shifts), image and pad slots ignored
    want = a["input_ids"].clone()
    want[a["image_token_mask"]] = -100
    n = 30 + 2 * 4
    want[n:] = -100
    assert torch.equal(a["labels"], want)
    assert a["image_grid_thw"].tolist() == [[1, 2, 2], [1, 2, 2]]
