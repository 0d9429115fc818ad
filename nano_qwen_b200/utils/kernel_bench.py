"""Per-kernel micro-benchmarks with roofline fractions.

    python -m nano_qwen_b200.utils.kernel_bench                 # every kernel, flagship shapes
    python -m nano_qwen_b200.utils.kernel_bench --only gemm_nt --iters 3   # small run for ncu

Shapes default to one Qwen3-1.7B training step's (4 x 4096 tokens, hidden
2048, 16/8 heads of 128, FFN 6144).  Each kernel is timed with CUDA events on
the launching stream after warm-up; the inputs of the memory-bound kernels are
larger than the 126 MB L2.  FLOP-bound kernels report TFLOP/s and the fraction
of the measured cuBLAS bf16 peak, memory-bound ones GB/s and the fraction of
the measured copy bandwidth (``MEASURED_PEAKS.json``).  Prints one JSON line
per kernel.
"""

from __future__ import annotations

import argparse
import json
import math
from typing import Callable, Dict, List

import torch

from .flops import measured_peaks


def _time(fn: Callable[[], None], iters: int, warmup: int = 3) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters * 1e-3


def cases(T: int, H: int, Hq: int, Hk: int, D: int, I: int, B: int, S: int) -> Dict[str, Callable]:
    from ..ops._ext import ext
    E = ext()
    dev = "cuda"
    out: Dict[str, Callable] = {}

    def gemm_nt():
        a = torch.randn(T, H, device=dev).bfloat16()
        w = torch.randn(2 * I, H, device=dev).bfloat16()
        return (lambda: E.gemm_nt(a, w)), 2.0 * T * H * 2 * I, None
    out["gemm_nt"] = gemm_nt

    def gemm_nt_swiglu():
        x = torch.randn(T, H, device=dev).bfloat16()
        w = (torch.randn(2 * I, H, device=dev) / math.sqrt(H)).bfloat16()
        return (lambda: E.gemm_nt_swiglu(x, w)), 2.0 * T * H * 2 * I, None
    out["gemm_nt_swiglu"] = gemm_nt_swiglu

    def gemm_nn():
        dy = torch.randn(T, 2 * I, device=dev).bfloat16()
        w = torch.randn(2 * I, H, device=dev).bfloat16()
        return (lambda: E.gemm_nn(dy, w)), 2.0 * T * H * 2 * I, None
    out["gemm_nn"] = gemm_nn

    def gemm_tn_acc():
        dy = torch.randn(T, 2 * I, device=dev).bfloat16()
        x = torch.randn(T, H, device=dev).bfloat16()
        c = torch.zeros(2 * I, H, device=dev)
        return (lambda: E.gemm_tn_acc(dy, x, c)), 2.0 * T * H * 2 * I, None
    out["gemm_tn_acc"] = gemm_tn_acc

    def _attn_inputs():
        qkv = (torch.randn(T, (Hq + 2 * Hk) * D, device=dev) * 0.5).bfloat16()
        qk = qkv[:, :(Hq + Hk) * D].contiguous()
        return qkv, qk

    attn_flops = 4.0 * B * Hq * D * S * S / 2  # causal

    def attn_fwd():
        qkv, qk = _attn_inputs()
        return (lambda: E.attn_fwd(qk, qkv, B, S, Hq, Hk, D, True, 1 / math.sqrt(D))), attn_flops, None
    out["attn_fwd"] = attn_fwd

    def attn_bwd():
        qkv, qk = _attn_inputs()
        o, lse = E.attn_fwd(qk, qkv, B, S, Hq, Hk, D, True, 1 / math.sqrt(D))
        do = torch.randn_like(o)
        dqkv = torch.empty_like(qkv)
        return (lambda: E.attn_bwd(do, qk, qkv, o, lse, dqkv, B, S, Hq, Hk, D, True,
                                   1 / math.sqrt(D))), 2.5 * attn_flops, None
    out["attn_bwd"] = attn_bwd

    def add_rmsnorm_fwd():
        x = torch.randn(T, H, device=dev)
        d = torch.randn(T, H, device=dev).bfloat16()
        w = torch.randn(H, device=dev)
        by = T * H * (4 + 2 + 4 + 2) + T * 4
        return (lambda: E.add_rmsnorm_fwd(x, d, w, 1e-6)), None, by
    out["add_rmsnorm_fwd"] = add_rmsnorm_fwd

    def add_rmsnorm_bwd():
        dy = torch.randn(T, H, device=dev).bfloat16()
        dh = torch.randn(T, H, device=dev)
        h = torch.randn(T, H, device=dev)
        w = torch.randn(H, device=dev)
        r = torch.rand(T, device=dev)
        dw = torch.zeros(H, device=dev)
        by = T * H * (2 + 4 + 4 + 4 + 2)
        return (lambda: E.add_rmsnorm_bwd(dy, dh, h, w, r, dw)), None, by
    out["add_rmsnorm_bwd"] = add_rmsnorm_bwd

    def _rope():
        qkv = torch.randn(T, (Hq + 2 * Hk) * D, device=dev).bfloat16()
        qw = torch.rand(D, device=dev)
        kw = torch.rand(D, device=dev)
        cos = torch.rand(S, D // 2, device=dev)
        sin = torch.rand(S, D // 2, device=dev)
        return qkv, qw, kw, cos, sin

    def qknorm_rope_fwd():
        qkv, qw, kw, cos, sin = _rope()
        by = T * (Hq + Hk) * D * 4
        return (lambda: E.qknorm_rope_fwd(qkv, qw, kw, cos, sin, None, B, S, Hq, Hk, D, 1e-6)), None, by
    out["qknorm_rope_fwd"] = qknorm_rope_fwd

    def qknorm_rope_bwd():
        qkv, qw, kw, cos, sin = _rope()
        _, rs = E.qknorm_rope_fwd(qkv, qw, kw, cos, sin, None, B, S, Hq, Hk, D, 1e-6)
        dqk = torch.randn(T, (Hq + Hk) * D, device=dev)
        dqkv = torch.empty_like(qkv)
        dqw = torch.zeros(D, device=dev)
        dkw = torch.zeros(D, device=dev)
        by = T * (Hq + Hk) * D * (4 + 2 + 2)
        return (lambda: E.qknorm_rope_bwd(dqk, qkv, qw, kw, rs, cos, sin, None, dqkv, dqw, dkw,
                                          B, S, Hq, Hk, D)), None, by
    out["qknorm_rope_bwd"] = qknorm_rope_bwd

    def swiglu_fwd():
        gu = torch.randn(T, 2 * I, device=dev).bfloat16()
        return (lambda: E.swiglu_fwd(gu)), None, T * I * 6
    out["swiglu_fwd"] = swiglu_fwd

    def swiglu_bwd():
        gu = torch.randn(T, 2 * I, device=dev).bfloat16()
        dh = torch.randn(T, I, device=dev).bfloat16()
        return (lambda: E.swiglu_bwd(dh, gu)), None, T * I * 10
    out["swiglu_bwd"] = swiglu_bwd

    def ce_fused_chunk():
        V = 151936
        R = 8192
        logits = (torch.randn(R, V, device=dev) * 3).bfloat16()
        labels = torch.randint(0, V, (R,), device=dev)
        nv = E.ce_count_valid(labels)
        ls = torch.zeros((), device=dev)
        return (lambda: E.ce_fused_chunk(logits, labels, nv, ls, True)), None, R * V * 4
    out["ce_fused_chunk"] = ce_fused_chunk

    def adamw_flat():
        n = 1 << 28
        p, g, m, v = (torch.randn(n, device=dev) for _ in range(4))
        comp = torch.empty(n, device=dev, dtype=torch.bfloat16)
        clip = torch.ones((), device=dev)
        return (lambda: E.adamw_flat(p, g, m, v, comp, clip, 0, n, 0, n, 1e-4, 1e-4, 0.9, 0.95, 1e-8,
                                     0.1, 0.1, 0.05)), None, n * (16 + 12 + 2)
    out["adamw_flat"] = adamw_flat
    return out


def main(argv: List[str] = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--only", nargs="*", default=None)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--tokens", type=int, default=16384)
    ap.add_argument("--batch", type=int, default=4)
    ap.add_argument("--hidden", type=int, default=2048)
    ap.add_argument("--heads", type=int, default=16)
    ap.add_argument("--kv-heads", type=int, default=8)
    ap.add_argument("--head-dim", type=int, default=128)
    ap.add_argument("--ffn", type=int, default=6144)
    a = ap.parse_args(argv)
    S = a.tokens // a.batch
    peaks = measured_peaks()
    tbl = cases(a.tokens, a.hidden, a.heads, a.kv_heads, a.head_dim, a.ffn, a.batch, S)
    for name, make in tbl.items():
        if a.only and name not in a.only:
            continue
        fn, flops, by = make()
        t = _time(fn, a.iters, a.warmup)
        rec = {"kernel": name, "us": round(t * 1e6, 2)}
        if flops:
            tf = flops / t / 1e12
            rec.update(tflops=round(tf, 1), frac_of_measured_bf16=round(tf / peaks["bf16_tflops"], 3))
        if by:
            gbs = by / t / 1e9
            rec.update(gb_s=round(gbs, 1), frac_of_measured_hbm=round(gbs / peaks["hbm_gbs"], 3))
        print(json.dumps(rec), flush=True)
        del fn
        torch.cuda.empty_cache()
    from ..ops._ext import ext
    assert ext().error_flag_read() == 0, "a kernel recorded an error"


if __name__ == "__main__":
    main()
