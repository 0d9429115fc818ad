"""GPU checks of the vision stack: the GELU kernel, patch embedding (im2col
GEMM), ViT, DeepStack, Merger and the whole Qwen3-VL model on the sm_100a
kernels, each against the fp32 CPU statement of the same module with the
same weights."""

import copy

import pytest
import torch

pytestmark = pytest.mark.gpu

VLG = dict(hidden_size=256, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
           head_dim=64, intermediate_size=512, vocab_size=4096, max_position_embeddings=1024,
           tie_word_embeddings=True, vision_enabled=True, vision_hidden_size=256,
           vision_num_hidden_layers=2, vision_num_attention_heads=4, vision_intermediate_size=512,
           vision_patch_size=8, vision_image_size=64, vision_num_channels=3,
           vision_deepstack_layers=[0], vision_merger_spatial_factor=2)


def _rel(a, b):
    a, b = a.detach().float().cpu(), b.detach().float().cpu()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


def _cfg():
    from nano_qwen_b200.config import ModelConfig
    return ModelConfig(**VLG)


def test_gelu_kernel_matches_fp32():
    from nano_qwen_b200 import ops
    torch.manual_seed(0)
    x = (torch.randn(1000, 512) * 3).cuda().bfloat16().requires_grad_(True)
    y = ops.gelu(x)
    dy = torch.randn_like(y)
    y.backward(dy)
    xf = x.detach().float().cpu().requires_grad_(True)
    yf = torch.nn.functional.gelu(xf)
    yf.backward(dy.float().cpu())
    assert _rel(y, yf) < 1e-2
    assert _rel(x.grad, xf.grad) < 1e-2


def _module_pair(make):
    torch.manual_seed(1)
    cpu = make()
    gpu = copy.deepcopy(cpu).cuda()
    return cpu, gpu


def _check_fwd_bwd(cpu, gpu, inputs_cpu, run, fwd_tol=2e-2, grad_tol=4e-2):
    outs_c = run(cpu, inputs_cpu)
    outs_g = run(gpu, [t.cuda() if torch.is_tensor(t) else t for t in inputs_cpu])
    g = torch.Generator().manual_seed(9)
    w = torch.randn(outs_c.shape, generator=g)
    (outs_c.float() * w).sum().backward()
    (outs_g.float() * w.cuda()).sum().backward()
    torch.cuda.synchronize()
    assert _rel(outs_g, outs_c) < fwd_tol, _rel(outs_g, outs_c)
    gp = dict(gpu.named_parameters())
    for n, p in cpu.named_parameters():
        if p.grad is None:
            continue
        assert gp[n].grad is not None, n
        assert _rel(gp[n].grad, p.grad) < grad_tol, (n, _rel(gp[n].grad, p.grad))


def test_patch_embedding_gemm_matches_conv():
    from nano_qwen_b200.models.vision.patch_embed import PatchEmbedding
    cpu, gpu = _module_pair(lambda: PatchEmbedding(_cfg()))
    x = torch.randn(3, 3, 64, 64)
    # the CPU statement here is the reference's Conv2d itself
    conv = lambda m, ins: torch.nn.functional.conv2d(ins[0], m.proj.weight, m.proj.bias, stride=8) \
        .flatten(2).transpose(1, 2) if not ins[0].is_cuda else m(ins[0])
    _check_fwd_bwd(cpu, gpu, [x], conv)


def test_vit_forward_backward_matches_fp32():
    from nano_qwen_b200.models.vision.vit import VisionTransformer
    cpu, gpu = _module_pair(lambda: VisionTransformer(_cfg()))

    def run(m, ins):
        o = m(ins[0])
        return torch.cat([o["last_hidden_state"].float()] + [s.float() for s in o["intermediate_states"]], 1)

    _check_fwd_bwd(cpu, gpu, [torch.randn(2, 3, 64, 64)], run)


def test_deepstack_and_merger_match_fp32():
    from nano_qwen_b200.models.vision.deepstack import DeepStack
    from nano_qwen_b200.models.vision.merger import VisionMerger
    cpu, gpu = _module_pair(lambda: DeepStack(256, 256, 2))
    with torch.no_grad():
        cpu.fusion_weights.copy_(torch.tensor([0.4, -0.3]))
        gpu.fusion_weights.copy_(cpu.fusion_weights)
    st = [torch.randn(2, 64, 256) for _ in range(2)]
    _check_fwd_bwd(cpu, gpu, st, lambda m, ins: m([ins[0]], ins[1]))
    cpu, gpu = _module_pair(lambda: VisionMerger(256, 256, 2))
    _check_fwd_bwd(cpu, gpu, [torch.randn(2, 64, 256)], lambda m, ins: m(ins[0], 8, 8))


def test_vl_model_loss_and_grads_match_cpu():
    """The whole Qwen3-VL model (MRoPE on) through the flat parameter store
    on the GPU against the fp32 CPU model with the same weights."""
    from nano_qwen_b200.models.multimodal import Qwen3VLModel
    from nano_qwen_b200.training.optimizer import attach_param_store
    torch.manual_seed(0)
    cpu = Qwen3VLModel(_cfg())
    gpu = copy.deepcopy(cpu).cuda()
    attach_param_store(gpu)
    g = torch.Generator().manual_seed(4)
    B, S = 2, 256
    ids = torch.randint(0, 4096, (B, S), generator=g)
    mask = torch.zeros(B, S, dtype=torch.bool)
    mask[0, 8:24] = True
    mask[1, 100:116] = True
    px = torch.randn(B, 3, 64, 64, generator=g)
    out = gpu(ids.cuda(), pixel_values=px.cuda(), image_token_mask=mask.cuda(), labels=ids.cuda())
    out["loss"].backward()
    torch.cuda.synchronize()
    ref = cpu(ids, pixel_values=px, image_token_mask=mask, labels=ids)
    ref["loss"].backward()
    assert abs(out["loss"].item() - ref["loss"].item()) < 2e-2 * ref["loss"].item()
    cp = dict(cpu.named_parameters())
    for n, p in gpu.named_parameters():
        if cp[n].grad is None or cp[n].grad.norm() == 0:
            continue
        assert _rel(p.grad, cp[n].grad) < 6e-2, (n, _rel(p.grad, cp[n].grad))
