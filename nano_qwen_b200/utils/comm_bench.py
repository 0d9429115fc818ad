"""Roofline benchmark of the peer-memory data-parallel kernels against NCCL.

    torchrun --nproc-per-node N -m nano_qwen_b200.utils.comm_bench [--numel 1.7e9]
    torchrun --nproc-per-node N -m nano_qwen_b200.utils.comm_bench --path ep
    torchrun --nproc-per-node N -m nano_qwen_b200.utils.comm_bench --path tp   # or cp

For a flat fp32 gradient of ``numel`` elements (default: the Qwen3-1.7B
store) it times, with CUDA events and the max over ranks:

* ``zero_rs`` (P2P reduce-scatter of the mean + squared norm) vs NCCL
  ``reduce_scatter_tensor`` (AVG) + a sum-of-squares kernel;
* ``zero_adamw_ag`` (sharded AdamW + bf16 all-gather by P2P stores) vs the
  AdamW kernel + NCCL ``all_gather_into_tensor``.

Roofline: the slower of (bytes that must cross NVLink into each GPU ÷ the
measured peer copy bandwidth, 770 GB/s per direction on this pool's B200s) and
(HBM bytes ÷ the measured copy bandwidth).  NVLink bytes: (N-1)/N x numel x 4
for the reduce-scatter, (N-1)/N x numel x 2 for the all-gather; the AdamW half
also moves 30 bytes per shard element through HBM.  Prints one JSON line per
path.
"""

from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

LINK_GBS = 770.0


def _timed(fn, iters: int, warmup: int = 3) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    t = torch.tensor([s.elapsed_time(e) / iters / 1e3], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t)


def ep_layer(iters: int, world: int, rank: int) -> None:
    """One expert-parallel MoE layer (the debug_moe shape: hidden 512, 64
    experts, top-8, expert FFN 256, 8 x 2048 tokens per rank), forward +
    backward, fused peer-memory path vs NCCL all-to-all.  Roofline: the slower
    of the expert GEMM FLOPs at the measured sustained bf16 peak and the token
    rows that must cross NVLink (dispatch + combine, and again in the
    backward: 4 x N*k*(W-1)/W rows of H bf16 per rank) at the link bandwidth."""
    from ..config import ModelConfig
    from ..models.moe import MoELayer
    from ..parallel.expert_parallel import apply_expert_parallel
    from ..training.optimizer import attach_param_store
    from .flops import measured_peaks
    cfg = ModelConfig(hidden_size=512, num_hidden_layers=1, num_attention_heads=8, num_key_value_heads=2,
                      head_dim=64, intermediate_size=1408, vocab_size=32000, num_experts=64,
                      num_experts_per_tok=8, moe_intermediate_size=256)
    N, H, K, I = 8 * 2048, 512, 8, 256
    grp = dist.new_group(list(range(world)))
    g = torch.Generator(device="cuda").manual_seed(3 + rank)
    x = torch.randn(N, H, device="cuda", generator=g).bfloat16()
    dy = torch.randn(N, H, device="cuda", generator=g).bfloat16()
    peak = measured_peaks().get("bf16_tflops_sustained", 1392.0) * 1e12
    flops = 3 * 2.0 * N * K * H * 2 * I + 3 * 2.0 * N * K * I * H  # gate|up and down, fwd + 2x bwd
    link = 4 * N * K * (world - 1) / world * H * 2
    for fused in (True, False):
        torch.manual_seed(0)

        class Wrap(torch.nn.Module):
            def __init__(self):
                super().__init__()
                self.moe = MoELayer(cfg)

        m = Wrap()
        with torch.no_grad():  # the module leaves its weights uninitialised; the model's init
            for p in m.parameters():
                p.normal_(0.0, 0.02)
        m = m.cuda()
        apply_expert_parallel(m, grp, fused=fused)
        attach_param_store(m)
        xr = x.clone().requires_grad_(True)

        def step():
            out, aux = m.moe(xr)
            out.backward(dy)

        t = _timed(step, iters)
        if rank == 0:
            t_roof = max(flops / peak, link / (LINK_GBS * 1e9))
            print(json.dumps({"path": "ep moe layer fwd+bwd (" + ("fused peer-memory" if fused else "nccl") + ")",
                              "n_gpus": world, "tokens_per_rank": N, "ms": round(t * 1e3, 3),
                              "roofline_ms": round(t_roof * 1e3, 3), "frac_of_roofline": round(t_roof / t, 3)}),
                  flush=True)


def _one_layer_model(cfg, seed: int = 0):
    from ..models import Qwen3Model
    torch.manual_seed(seed)
    with torch.device("cuda"):
        m = Qwen3Model(cfg)
    return m


def tp_block(iters: int, world: int, rank: int, tokens: int = 65536, seq: int = 8192) -> None:
    """One Qwen3-8B-shaped transformer block (vocabulary cut to 4096 so the
    block dominates) under tensor + sequence parallelism over every rank,
    forward + backward of ``tokens`` global tokens: the fused path (norms
    all-gathering into peer memory, GEMMs waiting per row tile, reduce-scatter
    epilogues) vs NCCL collectives.  Roofline: the slower of the block's
    training FLOPs / world at the measured sustained bf16 peak and the NVLink
    bytes into each GPU (two all-gathers and two reduce-scatters of the
    [tokens, hidden] bf16 stream forward, the same backward:
    8 x (W-1)/W x tokens x hidden x 2 bytes) at the link bandwidth."""
    from ..config import ModelConfig
    from ..parallel.manager import ParallelConfig, ParallelismManager
    from ..training.optimizer import attach_param_store
    from .flops import measured_peaks
    cfg = ModelConfig(hidden_size=4096, num_hidden_layers=1, num_attention_heads=32,
                      num_key_value_heads=8, head_dim=128, intermediate_size=12288, vocab_size=4096,
                      max_position_embeddings=seq, rope_theta=1e6, tie_word_embeddings=True)
    B = tokens // seq
    peak = measured_peaks().get("bf16_tflops_sustained", 1392.0) * 1e12
    flops = tokens * cfg.train_flops_per_token(seq) / world
    link = 8 * (world - 1) / world * tokens * cfg.hidden_size * 2
    g = torch.Generator().manual_seed(7)
    ids = torch.randint(0, cfg.vocab_size, (B, seq), generator=g).cuda()
    for fused in (True, False):
        pm = ParallelismManager(ParallelConfig(tp_size=world, tp_fused=None if fused else False))
        m = pm.apply_parallelism(_one_layer_model(cfg))
        attach_param_store(m)

        def step():
            out = m(ids, labels=ids)
            out["loss"].backward()

        t = _timed(step, iters)
        if rank == 0:
            t_roof = max(flops / peak, link / (LINK_GBS * 1e9))
            print(json.dumps({"path": "tp block fwd+bwd (" + ("fused peer-memory" if getattr(m, "tp_fused", False)
                                                              else "nccl") + ")",
                              "n_gpus": world, "tokens": tokens, "ms": round(t * 1e3, 3),
                              "roofline_ms": round(t_roof * 1e3, 3), "frac_of_roofline": round(t_roof / t, 3)}),
                  flush=True)
        del m
        torch.cuda.empty_cache()


def cp_layer(iters: int, world: int, rank: int, seq: int = 32768) -> None:
    """One Qwen3-1.7B-shaped layer (vocabulary cut to 4096) over one
    ``seq``-token sequence split by context parallelism over every rank,
    forward + backward: gathered k|v by peer-memory stores (allgather) vs the
    k|v ring.  Roofline: the slower of the training FLOPs / world at the
    measured sustained bf16 peak and the NVLink bytes into each GPU (the
    other ranks' k|v rows in bf16 forward, their fp32 dk|dv partials of this
    rank's rows backward)."""
    from ..config import ModelConfig
    from ..parallel.manager import ParallelConfig, ParallelismManager
    from ..training.optimizer import attach_param_store
    from .flops import measured_peaks
    cfg = ModelConfig(hidden_size=2048, num_hidden_layers=1, num_attention_heads=16,
                      num_key_value_heads=8, head_dim=128, intermediate_size=6144, vocab_size=4096,
                      max_position_embeddings=seq, rope_theta=1e6, tie_word_embeddings=True)
    peak = measured_peaks().get("bf16_tflops_sustained", 1392.0) * 1e12
    flops = seq * cfg.train_flops_per_token(seq) / world
    kv_row = 2 * cfg.num_key_value_heads * cfg.head_dim
    link = (world - 1) / world * seq * kv_row * (2 + 4)
    g = torch.Generator().manual_seed(7)
    ids = torch.randint(0, cfg.vocab_size, (1, seq), generator=g).cuda()
    for mode in ("allgather", "ring"):
        pm = ParallelismManager(ParallelConfig(cp_size=world, cp_mode=mode))
        m = pm.apply_parallelism(_one_layer_model(cfg))
        attach_param_store(m)

        def step():
            out = m(ids, labels=ids)
            out["loss"].backward()

        t = _timed(step, iters)
        if rank == 0:
            t_roof = max(flops / peak, link / (LINK_GBS * 1e9))
            print(json.dumps({"path": f"cp layer fwd+bwd ({mode})", "n_gpus": world, "seq": seq,
                              "ms": round(t * 1e3, 3), "roofline_ms": round(t_roof * 1e3, 3),
                              "frac_of_roofline": round(t_roof / t, 3)}), flush=True)
        del m
        torch.cuda.empty_cache()


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--numel", type=float, default=1.72e9)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--path", default="dp", choices=["dp", "ep", "tp", "cp"])
    a = ap.parse_args(argv)
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    world, rank = dist.get_world_size(), dist.get_rank()
    if a.path in ("ep", "tp", "cp"):
        {"ep": ep_layer, "tp": tp_block, "cp": cp_layer}[a.path](a.iters, world, rank)
        dist.barrier()
        dist.destroy_process_group()
        return
    from ..ops._ext import ext
    from ..parallel.data_parallel import shard_bounds
    from ..parallel.peer_dp import SymmetricAllocator
    E = ext()
    n = int(a.numel) // (64 * world) * (64 * world)
    alloc = SymmetricAllocator()
    dev = torch.device("cuda", local)
    grad = alloc(n, torch.float32, dev)
    comp = alloc(n, torch.bfloat16, dev)
    flags = alloc(16, torch.int32, dev)
    grad.normal_()
    torch.cuda.synchronize()
    pg, pc, pf = alloc.peer_ptrs(grad), alloc.peer_ptrs(comp), alloc.peer_ptrs(flags)
    b, e = shard_bounds(n, world, rank)
    sq = torch.zeros(1, device=dev)
    epoch = [0]

    def rs():
        epoch[0] += 1
        E.zero_rs(pg, pc, pf, rank, b, e, sq, epoch[0], 0, 1.0)

    master = torch.randn(n, device=dev)
    m = torch.zeros(n, device=dev)
    v = torch.zeros(n, device=dev)
    clip = torch.ones((), device=dev)

    def ag():
        E.zero_adamw_ag(pg, pc, pf, rank, master, m, v, clip, b, e, 0, e, 1e-4, 1e-4, 0.9, 0.95,
                        1e-8, 0.1, 0.1, 0.05)
        epoch[0] += 1
        E.zero_publish(pg, pc, pf, rank, epoch[0])

    plain = torch.randn(n, device=dev)
    out = torch.empty(n // world, device=dev)
    comp_plain = torch.empty(n, dtype=torch.bfloat16, device=dev)

    def nccl_rs():
        dist.reduce_scatter_tensor(out, plain, op=dist.ReduceOp.AVG)
        E.sum_squares(out)

    def nccl_ag():
        E.adamw_flat(master, plain, m, v, comp_plain, clip, b, e, 0, e, 1e-4, 1e-4, 0.9, 0.95, 1e-8,
                     0.1, 0.1, 0.05)
        dist.all_gather_into_tensor(comp_plain, comp_plain[b:e].clone())

    from .flops import measured_peaks
    hbm = measured_peaks()["hbm_gbs"]
    shard = n / world
    # (NVLink bytes into each GPU, HBM bytes on each GPU)
    rs_bytes = ((world - 1) / world * n * 4, n * 4 + shard * 4)
    ag_bytes = ((world - 1) / world * n * 2, shard * 30 + (world - 1) / world * n * 2)
    rows = [("zero_rs (P2P reduce-scatter + norm)", rs, rs_bytes),
            ("nccl reduce_scatter + sum_squares", nccl_rs, rs_bytes),
            ("zero_adamw_ag (AdamW + P2P all-gather)", ag, ag_bytes),
            ("adamw + nccl all_gather", nccl_ag, ag_bytes)]
    for name, fn, (link, mem) in rows:
        t = _timed(fn, a.iters)
        if rank == 0:
            t_roof = max(link / (LINK_GBS * 1e9), mem / (hbm * 1e9))
            print(json.dumps({"path": name, "n_gpus": world, "numel": n, "ms": round(t * 1e3, 3),
                              "nvlink_gb_s_per_gpu": round(link / t / 1e9, 1),
                              "roofline_ms": round(t_roof * 1e3, 3),
                              "frac_of_roofline": round(t_roof / t, 3)}), flush=True)
    assert E.error_flag_read() == 0, "kernel error word set"
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
