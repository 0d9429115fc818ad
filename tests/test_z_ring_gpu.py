"""The ring schedule's GPU pieces on one GPU: the flash-kernel chunk-pair
attention (full and causal pairs, forward and backward with a given output
and log-sum-exp) against its fp32 statement, and the QK-norm + RoPE
function against the CPU reference.  (The ring itself needs two or more
ranks: Gloo ranks on the CPU, ``tests/test_multi_gpu.py`` on GPUs.)"""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("D", [64, 128])
def test_kernel_pair_matches_fp32(causal, D):
    from nano_qwen_b200.parallel.ring_attention import KernelPair, TorchPair
    torch.manual_seed(0)
    B, c, Hq, Hk = 2, 256, 4, 2
    dev = torch.device("cuda", 0)
    q = torch.randn(B, c, Hq, D, device=dev).bfloat16()
    k = torch.randn(B, c, Hk, D, device=dev).bfloat16()
    v = torch.randn(B, c, Hk, D, device=dev).bfloat16()
    do = torch.randn(B, c, Hq, D, device=dev).bfloat16()
    scale = D ** -0.5
    o_k, lse_k = KernelPair().fwd(q, k, v, causal, scale)
    o_t, lse_t = TorchPair().fwd(q, k, v, causal, scale)
    torch.testing.assert_close(lse_k, lse_t, rtol=0, atol=2e-2)
    torch.testing.assert_close(o_k, o_t, rtol=0, atol=2e-2)
    grads_k = KernelPair().bwd(do, q, k, v, o_t.bfloat16(), lse_t, causal, scale)
    grads_t = TorchPair().bwd(do, q, k, v, o_t.bfloat16(), lse_t, causal, scale)
    for name, a, b in zip(("dq", "dk", "dv"), grads_k, grads_t):
        err = ((a.float() - b).norm() / b.norm()).item()
        assert err < 2e-2, (name, err)


def test_qknorm_rope_function_matches_reference():
    from nano_qwen_b200.models.rope import RotaryEmbedding
    from nano_qwen_b200.ops import reference as ref
    from nano_qwen_b200.parallel.ring_attention import _QKNormRope
    torch.manual_seed(0)
    B, S, Hq, Hk, D = 2, 128, 4, 2, 64
    dev = torch.device("cuda", 0)
    rope = RotaryEmbedding(D, 1024, 1e4)
    cos, sin = rope.cos_cached.to(dev), rope.sin_cached.to(dev)
    qkv = torch.randn(B, S, (Hq + 2 * Hk) * D, device=dev).bfloat16().requires_grad_(True)
    qw = torch.nn.Parameter(1 + 0.1 * torch.randn(D, device=dev))
    kw = torch.nn.Parameter(1 + 0.1 * torch.randn(D, device=dev))
    pos = torch.arange(S, device=dev).expand(B, S).contiguous()
    q, k, v = _QKNormRope.apply(qkv, qw, kw, cos, sin, pos, Hq, Hk, D, 1e-6)
    x = qkv.detach().float().cpu().requires_grad_(True)
    qr, kr, vr = x.split([Hq * D, Hk * D, Hk * D], -1)
    qw_c = qw.detach().cpu().requires_grad_(True)
    kw_c = kw.detach().cpu().requires_grad_(True)
    qr, kr = ref.qk_norm_rope(qr.reshape(B, S, Hq, D), kr.reshape(B, S, Hk, D), qw_c, kw_c,
                              cos.cpu()[pos.cpu()], sin.cpu()[pos.cpu()], 1e-6)
    torch.testing.assert_close(q.float().cpu(), qr, rtol=0, atol=3e-2)
    torch.testing.assert_close(k.float().cpu(), kr, rtol=0, atol=3e-2)
    gq, gk, gv = torch.randn_like(qr), torch.randn_like(kr), torch.randn(B, S, Hk, D)
    loss = (q.float() * gq.to(dev)).sum() + (k.float() * gk.to(dev)).sum() + (v.float() * gv.to(dev)).sum()
    loss.backward()
    (qr * gq).sum().add((kr * gk).sum()).add((vr.reshape(B, S, Hk, D) * gv).sum()).backward()
    err = ((qkv.grad.float().cpu() - x.grad).norm() / x.grad.norm()).item()
    assert err < 2e-2, err
