"""Numerics of every sm_100a kernel against a plain PyTorch fp32 statement of
the same op.  All tests here need a B200 and the built extension."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module")
def E():
    from nano_qwen_b200.ops import ext
    e = ext()
    e.error_flag_clear()
    yield e
    assert e.error_flag_read() == 0, "a kernel reported a bounded-wait timeout"


def rel_err(a, b):
    a = a.float()
    b = b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


# ----------------------------------------------------------------- GEMM
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 128), (200, 136, 72), (1000, 520, 1032),
                                   (4096, 2048, 2048)])
def test_gemm_nt(E, M, N, K):
    torch.manual_seed(0)
    A = torch.randn(M, K, device=DEV).bfloat16()
    B = torch.randn(N, K, device=DEV).bfloat16()
    C = E.gemm_nt(A, B)
    ref = A.float() @ B.float().t()
    assert rel_err(C, ref) < 1e-2


@pytest.mark.parametrize("M,I,K", [(128, 128, 64), (200, 256, 72), (1000, 384, 1032), (4096, 6144, 2048)])
def test_gemm_nt_swiglu(E, M, I, K):
    """GEMM with the SwiGLU epilogue: gu equals the plain GEMM bit for bit and
    h equals the separate SwiGLU kernel on that gu, and both match fp32."""
    torch.manual_seed(3)
    A = (torch.randn(M, K, device=DEV) * 0.5).bfloat16()
    W = (torch.randn(2 * I, K, device=DEV) / math.sqrt(K)).bfloat16()
    gu, h = E.gemm_nt_swiglu(A, W)
    assert torch.equal(gu, E.gemm_nt(A, W))
    assert torch.equal(h, E.swiglu_fwd(gu))
    ref = A.float() @ W.float().t()
    assert rel_err(gu, ref) < 1e-2
    g, u = ref.chunk(2, -1)
    assert rel_err(h, torch.nn.functional.silu(g) * u) < 1e-2


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 128), (200, 136, 72), (1000, 520, 1032)])
def test_gemm_nn(E, M, N, K):
    torch.manual_seed(1)
    A = torch.randn(M, K, device=DEV).bfloat16()
    B = torch.randn(K, N, device=DEV).bfloat16()
    C = E.gemm_nn(A, B)
    assert rel_err(C, A.float() @ B.float()) < 1e-2


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 128), (136, 200, 72), (520, 1000, 1032),
                                   (4096, 2048, 16384)])
def test_gemm_tn_acc(E, M, N, K):
    torch.manual_seed(2)
    A = torch.randn(K, M, device=DEV).bfloat16()
    B = torch.randn(K, N, device=DEV).bfloat16()
    C0 = torch.randn(M, N, device=DEV)
    C = C0.clone()
    E.gemm_tn_acc(A, B, C)
    ref = C0 + A.float().t() @ B.float()
    assert rel_err(C, ref) < 1e-2


@pytest.mark.parametrize("M,N,K", [(200, 136, 72), (1000, 520, 1032), (328, 2048, 256)])
def test_gemm_tma_epilogue_matches_register_epilogue(E, M, N, K):
    """The TMA-store epilogue (16-byte-aligned output rows) and the
    register-store epilogue (an output view whose row stride breaks TMA's
    16-byte rule) write the same bits, for bf16 stores and fp32 accumulation;
    row / column tails are clipped by the tensor map."""
    torch.manual_seed(5)
    A = torch.randn(M, K, device=DEV).bfloat16()
    B = torch.randn(N, K, device=DEV).bfloat16()
    c_tma = E.gemm_nt(A, B)
    wide = torch.zeros(M, N + 4, device=DEV).bfloat16()  # row stride 2N+8 bytes: register path
    E.gemm_nt_out(A, B, wide[:, :N])
    assert torch.equal(c_tma, wide[:, :N])
    assert not wide[:, N:].any()
    Bk = torch.randn(K, N, device=DEV).bfloat16()
    wide.zero_()
    E.gemm_nn_out(A, Bk, wide[:, :N])
    assert torch.equal(E.gemm_nn(A, Bk), wide[:, :N])
    At = torch.randn(K, M, device=DEV).bfloat16()
    c0 = torch.randn(M, N, device=DEV)
    c_tma = c0.clone()
    E.gemm_tn_acc(At, Bk, c_tma)
    widef = torch.zeros(M, N + 1, device=DEV)  # row stride 4N+4 bytes: register path
    widef[:, :N] = c0
    E.gemm_tn_acc(At, Bk, widef[:, :N])
    assert rel_err(c_tma, widef[:, :N]) < 1e-6  # fp32 adds in L2 vs in registers: same sums
    assert rel_err(c_tma, c0 + At.float().t() @ Bk.float()) < 1e-2


@pytest.mark.parametrize("M,N,K", [(2048, 4096, 512), (4096, 2048, 2048), (1000, 9000, 1032)])
def test_gemm_pair_kernels_match_one_sm(E, M, N, K):
    """The CTA-pair kernels (tcgen05.mma.cta_group::2, 256 x 256 tiles) write
    the same bits as the one-SM kernels for NT, NN, the SwiGLU epilogue and
    fp32 accumulation (same K order per output), and match fp32."""
    torch.manual_seed(6)
    A = torch.randn(M, K, device=DEV).bfloat16()
    B = torch.randn(N, K, device=DEV).bfloat16()
    Bk = torch.randn(K, N, device=DEV).bfloat16()
    W = (torch.randn(N // 256 * 256, K, device=DEV) / math.sqrt(K)).bfloat16()
    At = torch.randn(K, M, device=DEV).bfloat16()
    Bt = torch.randn(K, N // 8 * 8, device=DEV).bfloat16()
    c0 = torch.randn(M, N // 8 * 8, device=DEV)
    outs = {}
    before = E.gemm_pair_mode(-1)
    try:
        for mode in (1, 0):
            E.gemm_pair_mode(mode)
            c = c0.clone()
            E.gemm_tn_acc(At, Bt, c)
            outs[mode] = (E.gemm_nt(A, B), E.gemm_nn(A, Bk), E.gemm_nt_swiglu(A, W), c)
    finally:
        E.gemm_pair_mode(before)
    p, o = outs[1], outs[0]
    assert torch.equal(p[0], o[0]) and torch.equal(p[1], o[1])
    assert torch.equal(p[2][0], o[2][0]) and torch.equal(p[2][1], o[2][1])
    assert rel_err(p[3], o[3]) < 1e-6
    assert rel_err(p[0], A.float() @ B.float().t()) < 1e-2
    assert rel_err(p[1], A.float() @ Bk.float()) < 1e-2
    assert rel_err(p[3], c0 + At.float().t() @ Bt.float()) < 1e-2


def _grouped_inputs(G, R_per, K, seed=3):
    torch.manual_seed(seed)
    sizes = [R_per[g] for g in range(G)]
    offs = [0]
    for s in sizes:
        offs.append(offs[-1] + (s + 127) // 128 * 128)
    R = offs[-1] + 64
    X = torch.zeros(R, K, device=DEV).bfloat16()
    for g in range(G):
        X[offs[g]:offs[g] + sizes[g]] = torch.randn(sizes[g], K, device=DEV).bfloat16()
    return X, torch.tensor(offs, dtype=torch.int32, device=DEV), sizes, offs


def test_grouped_gemms(E):
    G, K, N = 4, 128, 192
    X, offs_t, sizes, offs = _grouped_inputs(G, [100, 0, 300, 129], K)
    W = torch.randn(G, N, K, device=DEV).bfloat16()
    Y = E.grouped_gemm_nt(X, W, offs_t)
    for g in range(G):
        a, b = offs[g], offs[g + 1]
        if b > a:
            assert rel_err(Y[a:b], X[a:b].float() @ W[g].float().t()) < 1e-2
    dY = torch.zeros_like(Y)
    for g in range(G):
        dY[offs[g]:offs[g] + sizes[g]] = torch.randn(sizes[g], N, device=DEV).bfloat16()
    dX = E.grouped_gemm_nn(dY, W, offs_t)
    for g in range(G):
        a, b = offs[g], offs[g + 1]
        if b > a:
            assert rel_err(dX[a:b], dY[a:b].float() @ W[g].float()) < 1e-2
    dW = torch.zeros(G, N, K, device=DEV)
    E.grouped_gemm_tn_acc(dY, X, dW, offs_t)
    for g in range(G):
        a, b = offs[g], offs[g + 1]
        ref = dY[a:b].float().t() @ X[a:b].float()
        if b > a:
            assert rel_err(dW[g], ref) < 1e-2
        else:
            assert dW[g].abs().max().item() == 0


# ---------------------------------------------------------------- norms
@pytest.mark.parametrize("H", [256, 2048, 4096])
def test_add_rmsnorm(E, H):
    torch.manual_seed(4)
    T = 300
    r = torch.randn(T, H, device=DEV)
    d = torch.randn(T, H, device=DEV).bfloat16()
    w = torch.rand(H, device=DEV) + 0.5
    h, y, rstd = E.add_rmsnorm_fwd(r, d, w, 1e-6)
    href = r + d.float()
    yref = href * torch.rsqrt(href.pow(2).mean(-1, keepdim=True) + 1e-6) * w
    assert rel_err(h, href) < 1e-6
    assert rel_err(y, yref) < 1e-2
    # backward vs autograd
    hr = href.clone().requires_grad_(True)
    wr = w.clone().requires_grad_(True)
    out = hr * torch.rsqrt(hr.pow(2).mean(-1, keepdim=True) + 1e-6) * wr
    dy = torch.randn(T, H, device=DEV).bfloat16()
    dh = torch.randn(T, H, device=DEV)
    out.backward(dy.float())
    dw = torch.zeros(H, device=DEV)
    dx, dxb = E.add_rmsnorm_bwd(dy, dh, h, w, rstd, dw)
    assert rel_err(dx, hr.grad + dh) < 1e-4
    assert rel_err(dw, wr.grad) < 1e-4


def test_layernorm(E):
    torch.manual_seed(5)
    T, H = 257, 1024
    x = torch.randn(T, H, device=DEV)
    w = torch.rand(H, device=DEV)
    b = torch.randn(H, device=DEV)
    y, mean, rstd = E.layernorm_fwd(x, w, b, 1e-5, torch.float32)
    xr = x.clone().requires_grad_(True)
    wr = w.clone().requires_grad_(True)
    br = b.clone().requires_grad_(True)
    yr = torch.nn.functional.layer_norm(xr, (H,), wr, br, 1e-5)
    assert rel_err(y, yr) < 1e-5
    dy = torch.randn(T, H, device=DEV)
    yr.backward(dy)
    dw = torch.zeros(H, device=DEV)
    db = torch.zeros(H, device=DEV)
    dx = E.layernorm_bwd(dy, x, w, mean, rstd, dw, db)
    assert rel_err(dx, xr.grad) < 1e-4
    assert rel_err(dw, wr.grad) < 1e-4
    assert rel_err(db, br.grad) < 1e-4


# ------------------------------------------------------- rope + attention
def _qkv(B, S, Hq, Hk, D, seed=6):
    torch.manual_seed(seed)
    return torch.randn(B * S, (Hq + 2 * Hk) * D, device=DEV).bfloat16()


def _ref_qknorm_rope(qkv, qw, kw, cos, sin, B, S, Hq, Hk, D, eps=1e-6):
    from nano_qwen_b200.ops import reference as R
    x = qkv.float().view(B, S, Hq + 2 * Hk, D)
    q, k, v = x[:, :, :Hq], x[:, :, Hq:Hq + Hk], x[:, :, Hq + Hk:]
    q, k = R.qk_norm_rope(q, k, qw, kw, cos[:S].unsqueeze(0), sin[:S].unsqueeze(0), eps)
    return q, k, v


def test_qknorm_rope(E):
    from nano_qwen_b200.models.rope import rope_tables
    B, S, Hq, Hk, D = 2, 100, 4, 2, 128
    qkv = _qkv(B, S, Hq, Hk, D)
    qw = torch.rand(D, device=DEV) + 0.5
    kw = torch.rand(D, device=DEV) + 0.5
    cos, sin = [t.to(DEV) for t in rope_tables(D, 256, 1e6)]
    qk, rstd = E.qknorm_rope_fwd(qkv, qw, kw, cos, sin, None, B, S, Hq, Hk, D, 1e-6)
    q, k, _ = _ref_qknorm_rope(qkv, qw, kw, cos, sin, B, S, Hq, Hk, D)
    assert rel_err(qk[:, :Hq * D].view(B, S, Hq, D), q) < 1e-2
    assert rel_err(qk[:, Hq * D:].view(B, S, Hk, D), k) < 1e-2
    # backward through autograd on the fp32 statement
    x = qkv.float().clone().requires_grad_(True)
    qwr = qw.clone().requires_grad_(True)
    kwr = kw.clone().requires_grad_(True)
    xx = x.view(B, S, Hq + 2 * Hk, D)

    def rn(t, w):
        return t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + 1e-6) * w

    def rot(t):
        c = cos[:S].view(1, S, 1, D // 2)
        s = sin[:S].view(1, S, 1, D // 2)
        a, b = t[..., :D // 2], t[..., D // 2:]
        return torch.cat([a * c - b * s, b * c + a * s], -1)

    qo = rot(rn(xx[:, :, :Hq], qwr))
    ko = rot(rn(xx[:, :, Hq:Hq + Hk], kwr))
    g = torch.randn(B * S, (Hq + Hk) * D, device=DEV)
    (qo.reshape(B * S, -1) * g[:, :Hq * D]).sum().backward(retain_graph=True)
    (ko.reshape(B * S, -1) * g[:, Hq * D:]).sum().backward()
    dqkv = torch.zeros_like(qkv)
    dqw = torch.zeros(D, device=DEV)
    dkw = torch.zeros(D, device=DEV)
    E.qknorm_rope_bwd(g, qkv, qw, kw, rstd, cos, sin, None, dqkv, dqw, dkw, B, S, Hq, Hk, D)
    assert rel_err(dqkv[:, :(Hq + Hk) * D], x.grad[:, :(Hq + Hk) * D]) < 2e-2
    assert rel_err(dqw, qwr.grad) < 2e-2
    assert rel_err(dkw, kwr.grad) < 2e-2


@pytest.mark.parametrize("B,S,Hq,Hk,D,causal", [(1, 128, 2, 1, 128, True), (2, 256, 4, 2, 128, True),
                                                (1, 200, 2, 2, 128, True), (2, 384, 8, 2, 64, False),
                                                (1, 1024, 2, 1, 128, True), (1, 192, 1, 1, 128, True),
                                                (2, 384, 4, 2, 128, False)])
def test_attention_fwd_bwd(E, B, S, Hq, Hk, D, causal):
    from nano_qwen_b200.ops import reference as R
    torch.manual_seed(7)
    qk = torch.randn(B * S, (Hq + Hk) * D, device=DEV).bfloat16()
    qkv = torch.randn(B * S, (Hq + 2 * Hk) * D, device=DEV).bfloat16()
    scale = 1.0 / math.sqrt(D)
    o, lse = E.attn_fwd(qk, qkv, B, S, Hq, Hk, D, causal, scale)
    q = qk[:, :Hq * D].float().view(B, S, Hq, D).requires_grad_(True)
    k = qk[:, Hq * D:].float().view(B, S, Hk, D).requires_grad_(True)
    v = qkv[:, (Hq + Hk) * D:].float().view(B, S, Hk, D).requires_grad_(True)
    oref, lref = R.attention_lse(q, k, v, causal=causal, scale=scale)
    assert rel_err(o.view(B, S, Hq, D), oref) < 2e-2
    assert (lse - lref).abs().max().item() < 2e-2
    do = torch.randn(B * S, Hq * D, device=DEV).bfloat16()
    oref.backward(do.float().view(B, S, Hq, D))
    dqkv = torch.zeros_like(qkv)
    dqk = E.attn_bwd(do, qk, qkv, o, lse, dqkv, B, S, Hq, Hk, D, causal, scale)
    assert rel_err(dqk[:, :Hq * D].view(B, S, Hq, D), q.grad) < 3e-2
    assert rel_err(dqk[:, Hq * D:].view(B, S, Hk, D), k.grad) < 3e-2
    assert rel_err(dqkv[:, (Hq + Hk) * D:].view(B, S, Hk, D), v.grad) < 3e-2


def _segments(B, S, cuts, left_pad=None):
    seg = torch.zeros(B, S, dtype=torch.int64)
    for b in range(B):
        for c in cuts[b]:
            seg[b, c:] += 1
    return seg


@pytest.mark.parametrize("S,D", [(640, 128), (640, 64), (1024, 128)])
def test_attention_key_range_mask(E, S, D):
    """Causal attention within per-token key ranges (packed documents, a
    left-padded row) against the fp32 statement with the same mask; block
    skipping and the element masks at document edges both matter here."""
    from nano_qwen_b200.ops import KeyRange
    from nano_qwen_b200.ops import reference as R
    torch.manual_seed(17)
    B, Hq, Hk = 3, 4, 2
    # row 0: documents at 0 / 100 / 300 / 301 / 520; row 1: 37 pad tokens then
    # one document; row 2: a single document (plain causal)
    seg = _segments(B, S, [[100, 300, 301, 520], [37], []]).to(DEV)
    kr = KeyRange.from_segments(seg)
    lo_ref = torch.stack([torch.tensor([int((seg[b, :i + 1] == seg[b, i]).nonzero()[0]) for i in range(S)])
                          for b in range(B)]).to(DEV)
    assert torch.equal(kr.kv_lo.long(), lo_ref)
    qk = torch.randn(B * S, (Hq + Hk) * D, device=DEV).bfloat16()
    qkv = torch.randn(B * S, (Hq + 2 * Hk) * D, device=DEV).bfloat16()
    scale = 1.0 / math.sqrt(D)
    o, lse = E.attn_fwd(qk, qkv, B, S, Hq, Hk, D, True, scale, kr.kv_lo.reshape(-1))
    q = qk[:, :Hq * D].float().view(B, S, Hq, D).requires_grad_(True)
    k = qk[:, Hq * D:].float().view(B, S, Hk, D).requires_grad_(True)
    v = qkv[:, (Hq + Hk) * D:].float().view(B, S, Hk, D).requires_grad_(True)
    oref = R.attention(q, k, v, causal=True, scale=scale, kv_lo=kr.kv_lo)
    assert rel_err(o.view(B, S, Hq, D), oref) < 2e-2
    do = torch.randn(B * S, Hq * D, device=DEV).bfloat16()
    oref.backward(do.float().view(B, S, Hq, D))
    dqkv = torch.zeros_like(qkv)
    dqk = E.attn_bwd(do, qk, qkv, o, lse, dqkv, B, S, Hq, Hk, D, True, scale, kr.q_hi.reshape(-1))
    assert rel_err(dqk[:, :Hq * D].view(B, S, Hq, D), q.grad) < 3e-2
    assert rel_err(dqk[:, Hq * D:].view(B, S, Hk, D), k.grad) < 3e-2
    assert rel_err(dqkv[:, (Hq + Hk) * D:].view(B, S, Hk, D), v.grad) < 3e-2
    # the unmasked kernel differs on the packed row: the mask is really applied
    o_plain, _ = E.attn_fwd(qk, qkv, B, S, Hq, Hk, D, True, scale)
    assert rel_err(o_plain.view(B, S, Hq, D)[0, 300:], oref[0, 300:]) > 0.1
    assert rel_err(o_plain.view(B, S, Hq, D)[2], oref[2]) < 2e-2


def test_model_document_mask_matches_separate_documents():
    """Model level: a packed row with document ids gives each document the
    logits it gets alone (positions restart per document)."""
    from nano_qwen_b200.config import ModelConfig
    from nano_qwen_b200.models import Qwen3Model
    from nano_qwen_b200.training.optimizer import attach_param_store
    torch.manual_seed(3)
    cfg = ModelConfig(hidden_size=256, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                      head_dim=64, intermediate_size=512, vocab_size=1024, max_position_embeddings=1024,
                      tie_word_embeddings=True)
    m = Qwen3Model(cfg).cuda()
    attach_param_store(m)
    a = torch.randint(0, 1024, (1, 200), device=DEV)
    b = torch.randint(0, 1024, (1, 312), device=DEV)
    packed = torch.cat([a, b], 1)
    doc = torch.cat([torch.zeros(1, 200), torch.ones(1, 312)], 1).long().to(DEV)
    pos = torch.cat([torch.arange(200), torch.arange(312)]).view(1, -1).to(DEV)
    with torch.no_grad():
        lp = m(packed, position_ids=pos, document_ids=doc)["logits"].float()
        la = m(a)["logits"].float()
        lb = m(b)["logits"].float()
    assert rel_err(lp[:, :200], la) < 2e-2
    assert rel_err(lp[:, 200:], lb) < 2e-2


def test_decode_attention(E):
    from nano_qwen_b200.ops import reference as R
    torch.manual_seed(8)
    B, Smax, Hq, Hk, D, Sq = 2, 700, 8, 2, 128, 3
    kc = torch.randn(B, Smax, Hk, D, device=DEV).bfloat16()
    vc = torch.randn(B, Smax, Hk, D, device=DEV).bfloat16()
    q = torch.randn(B, Sq, Hq, D, device=DEV).bfloat16()
    lens = torch.tensor([500, 650], dtype=torch.int32, device=DEV)
    start = lens - Sq
    out = E.decode_attn(q, kc, vc, lens, start, 1.0 / math.sqrt(D))
    for b in range(B):
        n = int(lens[b])
        ref = R.attention(q[b:b + 1].float(), kc[b:b + 1, :n].float(), vc[b:b + 1, :n].float(),
                          causal=True, q_offset=n - Sq)
        assert rel_err(out[b:b + 1], ref) < 2e-2


# ------------------------------------------------------------ elementwise
def test_swiglu(E):
    torch.manual_seed(9)
    gu = torch.randn(333, 2 * 688, device=DEV).bfloat16()
    h = E.swiglu_fwd(gu)
    g, u = gu.float().chunk(2, -1)
    assert rel_err(h, torch.nn.functional.silu(g) * u) < 1e-2
    x = gu.float().clone().requires_grad_(True)
    a, b = x.chunk(2, -1)
    dh = torch.randn(333, 688, device=DEV).bfloat16()
    (torch.nn.functional.silu(a) * b).backward(dh.float())
    assert rel_err(E.swiglu_bwd(dh, gu), x.grad) < 1e-2


def test_cross_entropy_chunks(E):
    torch.manual_seed(10)
    R_, V = 64, 32000
    logits = (torch.randn(R_, V, device=DEV) * 3).bfloat16()
    labels = torch.randint(0, V, (R_,), device=DEV)
    labels[::7] = -100
    ref = torch.nn.functional.cross_entropy(logits.float(), labels, ignore_index=-100, reduction="sum")
    nv = E.ce_count_valid(labels)
    ls = torch.zeros((), device=DEV)
    buf = logits.clone()
    E.ce_fused_chunk(buf, labels, nv, ls, True)
    assert abs(ls.item() - ref.item()) / ref.item() < 1e-3
    lf = logits.float().requires_grad_(True)
    torch.nn.functional.cross_entropy(lf, labels, ignore_index=-100).backward()
    assert rel_err(buf, lf.grad) < 2e-2


def test_embedding(E):
    torch.manual_seed(11)
    V, H = 1000, 256
    w = torch.randn(V, H, device=DEV)
    ids = torch.randint(0, V, (4, 50), device=DEV)
    out = E.embedding_fwd(ids, w)
    assert torch.equal(out.view(4, 50, H), w[ids])
    d = torch.randn(200, H, device=DEV)
    g = torch.zeros(V, H, device=DEV)
    E.embedding_bwd(ids, d, g)
    ref = torch.zeros(V, H, device=DEV).index_add_(0, ids.reshape(-1), d)
    assert rel_err(g, ref) < 1e-5


def test_adamw_flat(E):
    torch.manual_seed(12)
    n = 10_000 * 4
    p = torch.randn(n, device=DEV)
    g = torch.randn(n, device=DEV)
    m = torch.zeros(n, device=DEV)
    v = torch.zeros(n, device=DEV)
    comp = torch.empty(n, device=DEV, dtype=torch.bfloat16)
    pr = p.clone().requires_grad_(True)
    opt = torch.optim.AdamW([pr], lr=1e-2, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    pr.grad = g.clone()
    opt.step()
    clip = torch.ones((), device=DEV)
    E.adamw_flat(p, g, m, v, comp, clip, 0, n, 0, n, 1e-2, 1e-2, 0.9, 0.95, 1e-8, 0.1, 0.1, 0.05)
    assert rel_err(p, pr.detach()) < 1e-6
    assert rel_err(comp, pr.detach()) < 1e-2
    assert abs(E.sum_squares(g).item() - (g * g).sum().item()) / (g * g).sum().item() < 1e-5


def test_adamw_flat_shard_state(E):
    """Optimizer state held for a shard only (sbase = begin): the same update
    as full-size state over that range, and nothing outside it is touched."""
    torch.manual_seed(14)
    n, b, e = 4096 * 4, 1024 * 4, 3072 * 4
    p = torch.randn(n, device=DEV)
    g = torch.randn(n, device=DEV)
    clip = torch.full((), 0.5, device=DEV)
    full = [p.clone(), torch.randn(n, device=DEV).abs(), torch.rand(n, device=DEV)]
    shard = [p.clone(), full[1][b:e].clone(), full[2][b:e].clone()]
    cf = torch.empty(n, device=DEV, dtype=torch.bfloat16)
    cs = torch.zeros(n, device=DEV, dtype=torch.bfloat16)
    args = (2e-3, 1e-3, 0.9, 0.95, 1e-8, 0.1, 0.3, 0.2)
    E.adamw_flat(full[0], g, full[1], full[2], cf, clip, b, e, 0, 2 * n // 3, *args)
    E.adamw_flat(shard[0], g, shard[1], shard[2], cs, clip, b, e, b, 2 * n // 3, *args)
    assert torch.equal(shard[0], full[0])
    assert torch.equal(shard[1], full[1][b:e]) and torch.equal(shard[2], full[2][b:e])
    assert torch.equal(cs[b:e], cf[b:e]) and not cs[:b].any() and not cs[e:].any()
    with pytest.raises(Exception):
        E.adamw_flat(shard[0], g, shard[1], shard[2], cs, clip, b - 4, e, b, n, *args)


# ------------------------------------------------------------------- MoE
def test_router_nonfinite_logits_stay_in_range(E):
    """A row with a non-finite logit still routes to K distinct experts in
    [0, E) (no out-of-range index reaches the dispatch) and the error word
    records kErrBadArg; finite rows are unaffected."""
    torch.manual_seed(15)
    N, Ex, k = 64, 64, 8
    logits = torch.randn(N, Ex, device=DEV)
    logits[3, 5] = float("nan")
    logits[7, :] = float("inf")
    E.error_flag_clear()
    w, idx, counts, psum = E.router_fwd(logits.bfloat16(), k, True)
    torch.cuda.synchronize()
    assert E.error_flag_read() == 7
    E.error_flag_clear()
    assert int(idx.min()) >= 0 and int(idx.max()) < Ex
    for r in range(N):
        assert len(set(idx[r].tolist())) == k
    assert int(counts.sum()) == N * k
    ok = [r for r in range(N) if r not in (3, 7)]
    ref_idx = torch.topk(torch.softmax(logits.bfloat16().float()[ok], -1), k, -1).indices
    assert torch.equal(idx[ok].long().sort(-1).values, ref_idx.sort(-1).values)


def test_router_and_plan(E):
    from nano_qwen_b200.ops import reference as R
    torch.manual_seed(13)
    N, Ex, k = 1000, 64, 8
    logits = torch.randn(N, Ex, device=DEV)
    w, idx, counts, psum = E.router_fwd(logits, k, True)
    wr, ir, pr = R.router(logits, k, True)
    assert torch.equal(idx.long().sort(-1).values, ir.sort(-1).values)
    assert rel_err(w.sort(-1).values, wr.sort(-1).values) < 1e-5
    assert torch.equal(counts, torch.bincount(ir.reshape(-1), minlength=Ex).float())
    assert rel_err(psum, pr.sum(0)) < 1e-5
    # backward
    lr = logits.clone().requires_grad_(True)
    w2, _, p2 = R.router(lr, k, True)
    dw = torch.randn(N, k, device=DEV)
    dps = torch.randn(Ex, device=DEV)
    # align gradient columns with the kernel's top-k order
    order = torch.argsort(idx.long(), -1)
    order_r = torch.argsort(ir, -1)
    dw_ref = torch.empty_like(dw)
    dw_ref.scatter_(1, order_r, dw.gather(1, order))
    ((w2 * dw_ref).sum() + (p2.sum(0) * dps).sum()).backward()
    dl = E.router_bwd(logits, w, idx, dw, dps, True)
    assert rel_err(dl, lr.grad) < 1e-4
    # plan: stable counting sort with capacity
    cap = 100
    slot, offs, src = E.moe_plan(idx, Ex, cap, 128)
    flat = idx.reshape(-1).long()
    for e in range(0, Ex, 7):
        pos = (flat == e).nonzero().squeeze(-1)
        kept = pos[:cap]
        s = slot.reshape(-1)[kept]
        assert torch.equal(s.long(), offs[e].long() + torch.arange(len(kept), device=DEV))
        assert (slot.reshape(-1)[pos[cap:]] == -1).all()
        assert torch.equal(src[s.long()].long(), kept // k)


def test_moe_ffn_matches_loop(E):
    import importlib
    L = importlib.import_module("nano_qwen_b200.ops.linear")
    from nano_qwen_b200.ops.moe import _MoEFFNFn, _moe_ffn_cpu
    torch.manual_seed(14)
    N, H, I, Ex, k = 300, 256, 128, 8, 2
    x = torch.randn(N, H, device=DEV).bfloat16()
    logits = torch.randn(N, Ex, device=DEV)
    w, idx, _, _ = E.router_fwd(logits, k, True)
    Wgu = (torch.randn(Ex * 2 * I, H, device=DEV) * 0.05)
    Wd = (torch.randn(Ex * H, I, device=DEV) * 0.05)
    gref = L.WeightRef(Wgu.bfloat16(), torch.zeros_like(Wgu), [Wgu])
    dref = L.WeightRef(Wd.bfloat16(), torch.zeros_like(Wd), [Wd])
    out = _MoEFFNFn.apply(x, w, idx, gref, dref, Ex, I, -1, Wgu, Wd)
    g2 = L.WeightRef(Wgu.bfloat16().float().cpu(), torch.zeros_like(Wgu).cpu(), [Wgu.cpu()])
    d2 = L.WeightRef(Wd.bfloat16().float().cpu(), torch.zeros_like(Wd).cpu(), [Wd.cpu()])
    ref = _moe_ffn_cpu(x.float().cpu(), w.cpu(), idx.cpu(), g2, d2, Ex, I, None)
    assert rel_err(out.cpu(), ref) < 2e-2


# ------------------------------------------------- context-parallel attention
@pytest.mark.parametrize("rank", [0, 1])
def test_attention_cp_kernels_match_reference(E, rank):
    """attn_fwd_cp / attn_bwd_cp for one rank of a cp=2 zigzag split, against
    fp32 attention of that rank's queries over all keys (causal by position)."""
    torch.manual_seed(20 + rank)
    B, S_full, Hq, Hk, D, cp = 1, 2048, 4, 2, 128, 2
    c = S_full // (2 * cp)
    pos = torch.cat([torch.arange(rank * c, (rank + 1) * c),
                     torch.arange((2 * cp - 1 - rank) * c, (2 * cp - rank) * c)]).to(DEV)
    S = pos.numel()
    q = (torch.randn(B, S, Hq, D, device=DEV) * 0.5).bfloat16()
    k = (torch.randn(B, S_full, Hk, D, device=DEV) * 0.5).bfloat16()
    v = torch.randn(B, S_full, Hk, D, device=DEV).bfloat16()
    scale = 1.0 / math.sqrt(D)
    qk = torch.cat([q.reshape(B * S, Hq * D), torch.zeros(B * S, Hk * D, device=DEV).bfloat16()], 1).contiguous()
    kv = torch.cat([k.reshape(B * S_full, Hk * D), v.reshape(B * S_full, Hk * D)], 1).contiguous()
    o, lse = E.attn_fwd_cp(qk, kv, B, S, S_full, Hq, Hk, D, rank * c, (2 * cp - 1 - rank) * c, c, scale, 0, 0, cp)
    # reference
    qf = q.float().requires_grad_(True)
    kf = k.float().requires_grad_(True)
    vf = v.float().requires_grad_(True)
    g = Hq // Hk
    s = torch.einsum("bqhd,bkhd->bhqk", qf, kf.repeat_interleave(g, 2)) * scale
    mask = torch.arange(S_full, device=DEV)[None, :] > pos[:, None]
    s = s.masked_fill(mask, float("-inf"))
    p = torch.softmax(s, -1)
    ref = torch.einsum("bhqk,bkhd->bqhd", p, vf.repeat_interleave(g, 2))
    assert rel_err(o.view(B, S, Hq, D), ref) < 2e-2
    do = torch.randn(B, S, Hq, D, device=DEV).bfloat16()
    ref.backward(do.float())
    dqk, dkv = E.attn_bwd_cp(do.reshape(B * S, Hq * D).contiguous(), qk, kv, o, lse, B, S, S_full, Hq, Hk, D,
                             rank * c, (2 * cp - 1 - rank) * c, c, scale, None)
    assert rel_err(dqk[:, :Hq * D].view(B, S, Hq, D), qf.grad) < 3e-2
    assert rel_err(dkv[:, :Hk * D].view(B, S_full, Hk, D), kf.grad) < 3e-2
    assert rel_err(dkv[:, Hk * D:].view(B, S_full, Hk, D), vf.grad) < 3e-2
    assert E.error_flag_read() == 0
