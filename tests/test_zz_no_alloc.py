"""The allocation-free decode-attention entry point, called through its
exported C symbol, against the regular ``decode_attn`` binding.

Named to be collected last, so that it also runs after every other test has
used the library in the same process.
"""

import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel_err(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


def _entry():
    from nano_qwen_b200 import _C  # noqa: F401  (loads the library)
    lib = ctypes.CDLL(_C.__file__)
    fn = lib.nq_decode_attn_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int] * 6 + [ctypes.c_float, ctypes.c_void_p,
                                                                ctypes.c_char_p, ctypes.c_int]
    return fn


def _call(fn, q, kc, vc, lens, start, out, scale):
    B, Sq, Hq, D = q.shape
    Smax, Hk = kc.shape[1], kc.shape[2]
    err = ctypes.create_string_buffer(256)
    rc = fn(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), lens.data_ptr(), start.data_ptr(),
            out.data_ptr(), B, Sq, Hq, Hk, D, Smax, scale,
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), err, len(err))
    return rc, err.value.decode()


def _case(seed, B, Smax, Hq, Hk, D, Sq, lens):
    g = torch.Generator(device="cuda").manual_seed(seed)
    kc = torch.randn(B, Smax, Hk, D, device="cuda", generator=g).bfloat16()
    vc = torch.randn(B, Smax, Hk, D, device="cuda", generator=g).bfloat16()
    q = torch.randn(B, Sq, Hq, D, device="cuda", generator=g).bfloat16()
    lens = torch.tensor(lens, dtype=torch.int32, device="cuda")
    return q, kc, vc, lens, (lens - Sq).to(torch.int32)


def _oracle(q, kc, vc, lens, start, scale):
    """fp32 statement of decode attention: query row i of sequence b sits at
    position start[b] + i and sees cache rows j <= that position (j < lens[b]);
    query head h reads kv head h // (Hq / Hk)."""
    B, Sq, Hq, D = q.shape
    g = Hq // kc.shape[2]
    out = torch.empty(B, Sq, Hq, D, dtype=torch.float32, device=q.device)
    for b in range(B):
        L, s0 = int(lens[b]), int(start[b])
        k = kc[b, :L].float().repeat_interleave(g, dim=1)
        v = vc[b, :L].float().repeat_interleave(g, dim=1)
        s = torch.einsum("qhd,khd->hqk", q[b].float(), k) * scale
        pos = s0 + torch.arange(Sq, device=q.device)[:, None]
        s = s.masked_fill(torch.arange(L, device=q.device)[None, :] > pos, float("-inf"))
        out[b] = torch.einsum("hqk,khd->qhd", s.softmax(-1), v)
    return out


def test_noalloc_matches_decode_attn_two_calls():
    """Two calls in a row on one stream, with different shapes (so the second
    reuses the shared scratch with another layout), before any sync.  Both
    must equal ``decode_attn`` bit for bit (same kernels, same split choice)
    and match the fp32 statement of attention."""
    from nano_qwen_b200.ops._ext import ext
    fn = _entry()
    cases = [(11, 2, 700, 8, 2, 128, 3, [500, 650]),
             (12, 3, 1024, 16, 8, 64, 1, [1, 1000, 517])]
    for order in (cases, cases[::-1]):
        runs = []
        for seed, B, Smax, Hq, Hk, D, Sq, lens in order:
            q, kc, vc, ln, st = _case(seed, B, Smax, Hq, Hk, D, Sq, lens)
            scale = 1.0 / math.sqrt(D)
            out = torch.full_like(q, float("nan"))
            rc, msg = _call(fn, q, kc, vc, ln, st, out, scale)
            assert rc == 0, msg
            runs.append((q, kc, vc, ln, st, scale, out))
        torch.cuda.synchronize()
        for q, kc, vc, ln, st, scale, out in runs:
            ref = ext().decode_attn(q, kc, vc, ln, st, scale)
            torch.cuda.synchronize()
            assert torch.equal(out, ref)
            assert _rel_err(out, _oracle(q, kc, vc, ln, st, scale)) < 1e-2


def test_noalloc_rejects_oversized_request():
    fn = _entry()
    # 512 sequences x 32 heads, one split each: 16384 rows * 130 floats > 8 MiB
    q, kc, vc, ln, st = _case(13, 512, 16, 32, 1, 128, 1, [16] * 512)
    out = torch.empty_like(q)
    rc, msg = _call(fn, q, kc, vc, ln, st, out, 0.1)
    assert rc != 0 and "scratch" in msg
