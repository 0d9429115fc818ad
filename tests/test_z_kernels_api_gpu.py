"""The reference-named kernel API on the GPU: its kernel-backed entries
(cross-entropy, flash attention, RMSNorm, SwiGLU) against fp32 PyTorch,
values and gradients."""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


def test_reference_kernel_api_on_gpu():
    from nano_qwen_b200 import kernels as K
    torch.manual_seed(0)
    dev = torch.device("cuda", 0)
    logits = torch.randn(256, 512, device=dev).bfloat16().requires_grad_(True)
    labels = torch.randint(0, 512, (256,), device=dev)
    labels[::7] = -100
    loss = K.fused_cross_entropy(logits, labels)
    loss.backward()
    x = logits.detach().float().requires_grad_(True)
    ref = F.cross_entropy(x, labels)
    ref.backward()
    assert abs(float(loss) - float(ref)) < 2e-2 * float(ref)
    assert _rel(logits.grad, x.grad) < 2e-2
    q = torch.randn(2, 8, 256, 128, device=dev).bfloat16().requires_grad_(True)
    k = torch.randn(2, 2, 256, 128, device=dev).bfloat16().requires_grad_(True)
    v = torch.randn(2, 2, 256, 128, device=dev).bfloat16().requires_grad_(True)
    o = K.flash_attention(q, k, v, causal=True)
    o.float().square().sum().backward()
    qf, kf, vf = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    of = F.scaled_dot_product_attention(qf, kf.repeat_interleave(4, 1), vf.repeat_interleave(4, 1),
                                        is_causal=True)
    of.square().sum().backward()
    assert _rel(o, of) < 2e-2
    for a, b in ((q.grad, qf.grad), (k.grad, kf.grad), (v.grad, vf.grad)):
        assert _rel(a, b) < 3e-2
    h = torch.randn(64, 256, device=dev).bfloat16()
    w = torch.rand(256, device=dev) + 0.5
    hn = K.rmsnorm(h, w, 1e-6)
    hf = h.float() * torch.rsqrt(h.float().pow(2).mean(-1, keepdim=True) + 1e-6) * w
    assert _rel(hn, hf) < 1e-2
    gate, up = torch.randn(64, 256, device=dev).bfloat16(), torch.randn(64, 256, device=dev).bfloat16()
    assert _rel(K.fused_swiglu(gate, up), F.silu(gate.float()) * up.float()) < 1e-2
