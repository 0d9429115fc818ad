"""The reference's standalone kernel API (``nano_qwen_b200.kernels``) against
the reference's own PyTorch fallbacks (installed copy under
``baseline/_ref``), on CPU."""

import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")
pytestmark = pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "kernels")),
                                reason="reference copy not present")


def _ref(name):
    if REF not in sys.path:
        sys.path.append(REF)
    import importlib
    return importlib.import_module(f"kernels.{name}")


def test_reference_kernel_api_matches_reference_fallbacks():
    from nano_qwen_b200 import kernels as K
    torch.manual_seed(0)
    # cross-entropy with ignored rows
    logits = torch.randn(12, 40)
    labels = torch.randint(0, 40, (12,))
    labels[3] = -100
    ce = _ref("cross_entropy")
    torch.testing.assert_close(K.fused_cross_entropy(logits, labels),
                               ce.fused_cross_entropy(logits, labels, use_triton=False))
    labels7 = torch.randint(0, 40, (12,))
    labels7[5] = 7
    torch.testing.assert_close(K.fused_cross_entropy(logits, labels7, ignore_index=7),
                               ce.fused_cross_entropy(logits, labels7, ignore_index=7, use_triton=False))
    # attention (same heads, causal and not)
    q, k, v = (torch.randn(2, 4, 16, 8) for _ in range(3))
    fa = _ref("flash_attn")
    for causal in (True, False):
        torch.testing.assert_close(K.flash_attention(q, k, v, causal=causal),
                                   fa.flash_attention(q, k, v, causal=causal, use_triton=False))
    # MoE scatter / gather
    md = _ref("moe_dispatch")
    x = torch.randn(10, 6)
    idx = torch.randperm(20).view(10, 2)   # one slot per (token, choice), as the dispatch uses it
    w = torch.rand(10, 2)
    torch.testing.assert_close(K.scatter_tokens(x, idx, w, 20),
                               md.scatter_tokens(x, idx, w, 20, use_triton=False))
    eo = torch.randn(20, 6)
    torch.testing.assert_close(K.gather_tokens(eo, idx, w, 10, 6),
                               md.gather_tokens(eo, idx, w, 10, 6, use_triton=False))
    # RMSNorm, RoPE, SwiGLU
    rn = _ref("rmsnorm")
    h = torch.randn(5, 32)
    wt = torch.rand(32) + 0.5
    torch.testing.assert_close(K.rmsnorm(h, wt, 1e-6), rn.pytorch_rmsnorm(h, wt, 1e-6))
    mod = K.FusedRMSNorm(32)
    torch.testing.assert_close(mod(h), rn.FusedRMSNorm(32, use_triton=False)(h))
    rp = _ref("rope")
    cos, sin = torch.rand(16, 4), torch.rand(16, 4)
    for a, b in zip(K.apply_rope(q, k, cos, sin), rp.apply_rope(q, k, cos, sin, use_triton=False)):
        torch.testing.assert_close(a, b)
    cos3, sin3 = torch.rand(2, 16, 4), torch.rand(2, 16, 4)
    for a, b in zip(K.apply_rope(q, k, cos3, sin3), rp.apply_rope(q, k, cos3, sin3, use_triton=False)):
        torch.testing.assert_close(a, b)
    sw = _ref("swiglu")
    gate, up = torch.randn(4, 24), torch.randn(4, 24)
    torch.testing.assert_close(K.fused_swiglu(gate, up), sw.fused_swiglu(gate, up, use_triton=False))
