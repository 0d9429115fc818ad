"""Headline benchmark: train tokens/s (device-timed, max over ranks) + MFU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config NAME]

Multi-GPU: launched by ``torch.distributed.run --nproc-per-node N``; each rank
reads RANK/LOCAL_RANK/WORLD_SIZE from the environment and uses NCCL.

Default config = the reference's functional headline path: Qwen3-1.7B-shaped
dense model (28 layers, hidden 2048, 16 Q / 8 KV heads, head_dim 128,
intermediate 6144, vocab 151936, tied embeddings), per-GPU batch 4 x 4096
uniform-random token ids, random-init weights, bf16 compute, AdamW with grad
clipping, data parallel over N GPUs (weak scaling).  ``--impl reference`` runs
the unmodified reference (``baseline/_ref``) through its own public API: its
``Qwen3Model`` + ``build_optimizer`` + ``build_scheduler`` under bf16 autocast
with ``clip_grad_norm_``, and for N>1 its ``ParallelismManager`` (FSDP2).

Timing: W untimed warm-up steps, then K steps bracketed by a barrier and
``torch.cuda.synchronize()`` on both sides, timed with CUDA events on the
launching stream; the per-step time is the max over ranks.  The step's working
set (3.4 GB of bf16 weights, tens of GB of activations) is far larger than the
126 MB L2, so no L2 flush is needed.  SM clocks and throttle reasons are
sampled with nvidia-smi during the timed region.  The end-to-end number ("e2e")
repeats the measurement through the public training API with, every step, a
pinned host->device copy of the step's token ids/labels and a device->host read
of the loss and grad norm, timed by the host clock.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))

DP_LABEL = {"p2p": "ZeRO-2, fused peer-memory reduce-scatter + sharded AdamW + all-gather kernels",
            "shard": "ZeRO-2 over NCCL reduce-scatter / all-gather",
            "replicate": "NCCL all-reduce",
            "fsdp": "fully sharded: per-block bf16 all-gather / fp32 reduce-scatter over NCCL"}

BASELINE_METRIC = "train tokens/sec (device-timed, max over ranks) at 1/2/4/8 B200; MFU"
# the reference's only published measurement: its CPU fp32 step of the debug model
CPU_BASELINE_TOKS = 1169.0

def load_configs(directory=None):
    """Benchmark configurations from ``configs/bench/*.yaml``:
    name -> (model kwargs, per-GPU micro batch, sequence length, parallel
    label: dp / tp / ep / cp)."""
    import glob
    import yaml
    directory = directory or os.path.join(os.path.dirname(os.path.abspath(__file__)), "configs", "bench")
    out = {}
    for path in sorted(glob.glob(os.path.join(directory, "*.yaml"))):
        with open(path) as f:
            d = yaml.safe_load(f)
        out[d["name"]] = (dict(d["model"]), int(d["micro_batch"]), int(d["seq_len"]), d["parallel"])
    return out


CONFIGS = load_configs()


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--config", default="qwen3-1.7b", choices=sorted(CONFIGS))
    p.add_argument("--e2e-steps", type=int, default=None)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--kernel-table", default=None,
                   help="ours: write per-kernel device time of the profiled extra step (markdown) to this path")
    p.add_argument("--overlap", action="store_true",
                   help="ours, dp p2p or shard: reduce-scatter per block during the backward instead of after it")
    p.add_argument("--comm", default="fused", choices=["fused", "nccl"],
                   help="ours, tp/ep configs: peer-memory fused kernels or NCCL collectives")
    p.add_argument("--dp-mode", default=None, choices=["p2p", "shard", "replicate", "fsdp"],
                   help="ours, N>1: peer-memory fused ZeRO step (p2p; the default for plain data "
                        "parallelism, opt-in under tp/ep/cp), NCCL ZeRO-2 / all-reduce, "
                        "or fully sharded parameters (fsdp)")
    p.add_argument("--cp-mode", default="allgather", choices=["allgather", "ring"],
                   help="ours, cp configs: gathered k|v (peer-memory kernels) or the k|v ring")
    p.add_argument("--device", default="cuda", choices=["cuda", "cpu"],
                   help="cpu: fp32 on the host, world size 1 (the reference's CPU debug step with --config debug)")
    return p.parse_args()


# ------------------------------------------------------------------ clocks
class ClockSampler:
    REASONS = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.idx)],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        def pump():
            for line in self.proc.stdout:
                self.lines.append(line.strip())
        self.thread = threading.Thread(target=pump, daemon=True)
        self.thread.start()

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=2)
        sm, mx, reasons = [], None, set()
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(self.REASONS, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ common
DEVICE = "cuda"  # --device


def dist_setup():
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if DEVICE == "cuda":
        torch.cuda.set_device(local)
    return world, rank, local


def maybe_init_pg(world, local):
    import datetime

    import torch
    import torch.distributed as dist
    if world > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))


def max_over_ranks(x: float) -> float:
    import torch
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())
    return x


def barrier():
    import torch
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        dist.barrier(device_ids=[torch.cuda.current_device()])


def flops_per_token(mk: dict, seq: int) -> float:
    h = mk["hidden_size"]
    L = mk["num_hidden_layers"]
    qd = mk["num_attention_heads"] * mk["head_dim"]
    kvd = mk["num_key_value_heads"] * mk["head_dim"]
    attn = h * qd * 2 + 2 * h * kvd
    if mk.get("num_experts"):
        ffn = mk["num_experts_per_tok"] * 3 * h * mk["moe_intermediate_size"] + h * mk["num_experts"]
    else:
        ffn = 3 * h * mk["intermediate_size"]
    n_active = L * (attn + ffn) + mk["vocab_size"] * h
    return 6.0 * n_active + 12.0 * L * qd * (seq / 2)


def measured_peak() -> float:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"]) * 1e12
    except Exception:
        return 1.59e15


def synthetic_batches(n, B, S, V, device, seed=1234, pinned=False):
    import torch
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(n):
        ids = torch.randint(0, V, (B, S), generator=g)
        if pinned:
            ids = ids.pin_memory()
        elif device is not None:
            ids = ids.to(device)
        out.append(ids)
    return out


def timed_loop(step_fn, inputs, K, W, local):
    """Warm-up W, then K device-timed steps; returns ms/step (max over ranks) and clocks."""
    import torch
    if DEVICE == "cpu":  # host-timed (fp32 on the CPU, one process)
        for i in range(W):
            step_fn(inputs[i % len(inputs)])
        t0 = time.perf_counter()
        for i in range(K):
            step_fn(inputs[i % len(inputs)])
        return (time.perf_counter() - t0) * 1e3 / K, {"sm_mhz": None, "sm_max_mhz": None,
                                                       "reasons": ["cpu run"]}
    for i in range(W):
        step_fn(inputs[i % len(inputs)])
    barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    e0.record()
    for i in range(K):
        step_fn(inputs[i % len(inputs)])
    e1.record()
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1) / K
    return max_over_ranks(ms), clocks


# ------------------------------------------------------------- our engine
def run_ours(args, world, rank, local):
    import torch
    sys.path.insert(0, ROOT)
    from nano_qwen_b200.config import ModelConfig
    from nano_qwen_b200.models import Qwen3Model
    from nano_qwen_b200.ops import ext
    from nano_qwen_b200.parallel.comm import init_distributed
    from nano_qwen_b200.training.engine import TrainEngine

    mk, B, S, par = CONFIGS[args.config]
    init_distributed()
    dev = torch.device("cuda", local) if DEVICE == "cuda" else torch.device("cpu")
    torch.manual_seed(0)
    cfg = ModelConfig(**mk)
    with torch.device(dev):
        model = Qwen3Model(cfg)
    tcfg = {"optimizer": {"lr": 3e-4, "weight_decay": 0.1, "grad_clip": 1.0},
            "scheduler": {"type": "cosine", "warmup_steps": 100, "total_steps": 100000},
            "distributed": {"fsdp_enabled": True, "overlap_grad_reduce": args.overlap}}
    pm = None
    if par in ("tp", "ep", "cp") and world > 1:
        from nano_qwen_b200.parallel.manager import ParallelConfig, ParallelismManager
        fused = None if args.comm == "fused" else False
        pm = ParallelismManager(ParallelConfig(tp_size=world if par == "tp" else 1,
                                               ep_size=world if par == "ep" else 1,
                                               cp_size=world if par == "cp" else 1,
                                               cp_mode=args.cp_mode,
                                               tp_fused=fused, ep_fused=fused))
        model = pm.apply_parallelism(model)
    eng = TrainEngine(model, tcfg, dev, dp_mode=args.dp_mode if world > 1 else None, parallel=pm)
    del model
    # tensor parallelism: every rank sees the same global batch
    seed_rank = 0 if par in ("tp", "cp") else rank
    inputs = synthetic_batches(4, B, S, cfg.vocab_size, dev, seed=1234 + seed_rank)

    def step(ids):
        eng.train_step([{"input_ids": ids, "labels": ids}])

    if DEVICE == "cpu":
        ms, clocks = timed_loop(step, inputs, args.steps, args.warmup, local)
        return ms, clocks, {"kernel_error_flag": 0, "gpu_launches_per_step": {"ours": 0, "all": 0},
                            "dp_mode": None}, None
    ext().error_flag_clear()
    ms, clocks = timed_loop(step, inputs, args.steps, args.warmup, local)
    err = ext().error_flag_read()
    launches = count_launches(step, inputs[0])
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e_ours(eng, args, B, S, cfg.vocab_size, dev, rank)
    mode = None
    if eng.dp is not None:
        mode = "p2p" if hasattr(eng.dp, "fused_step") else eng.dp.mode
    dp_step = mode
    if par == "tp" and world > 1:
        mode = "tp-fused" if getattr(eng.model, "tp_fused", False) else "tp-nccl"
    if par == "ep" and world > 1:
        eps = [m.ep for m in eng.model.modules() if getattr(m, "ep", None) is not None]
        mode = "ep-fused" if eps and all(e.fused for e in eps) else "ep-nccl"
    if par == "cp" and world > 1:
        mode = "cp-" + args.cp_mode
    return ms, clocks, {"kernel_error_flag": err, "gpu_launches_per_step": launches,
                        "dp_mode": mode, "dp_step": dp_step}, e2e


def count_launches(step_fn, ids):
    """Kernels of this repository (namespace nq::) launched by one training step,
    counted with the CUDA profiler on an extra, untimed step."""
    import torch
    from torch.profiler import ProfilerActivity, profile
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step_fn(ids)
        torch.cuda.synchronize()
    ours = total = 0
    per_kernel = {}
    spans = []
    for ev in prof.events():
        if ev.device_type is not None and str(ev.device_type).endswith("CUDA"):
            total += 1
            if "nq::" in ev.name:
                ours += 1
            a = per_kernel.setdefault(ev.name, [0, 0.0])
            a[0] += 1
            a[1] += getattr(ev, "device_time_total", 0.0)
            tr = getattr(ev, "time_range", None)
            if tr is not None:
                spans.append((tr.start, tr.end))
    if KERNEL_TABLE:
        write_kernel_table(KERNEL_TABLE, per_kernel, spans)
    return {"ours": ours, "all": total}


KERNEL_TABLE = None  # --kernel-table PATH (rank 0)


def write_kernel_table(path, per_kernel, spans=()):
    """Device time per kernel over the profiled (untimed) step, largest first,
    and the device time with no kernel running (union of the kernels'
    intervals against first start .. last end).  Profiler timestamps: use the
    shares, not the absolute step time."""
    tot = sum(t for _, t in per_kernel.values()) or 1.0
    busy = idle = 0.0
    if spans:
        spans = sorted(spans)
        cur_s, cur_e = spans[0]
        for s0, e0 in spans[1:]:
            if s0 > cur_e:
                busy += cur_e - cur_s
                cur_s, cur_e = s0, e0
            else:
                cur_e = max(cur_e, e0)
        busy += cur_e - cur_s
        idle = max(e for _, e in spans) - spans[0][0] - busy
    with open(path, "w") as f:
        f.write(f"# one training step, kernel device time total {tot / 1e3:.1f} ms\n")
        if spans:
            f.write(f"# device busy {busy / 1e3:.1f} ms, idle between kernels {idle / 1e3:.1f} ms\n")
        f.write("| kernel | launches | ms | share |\n|---|---|---|---|\n")
        for name, (n, t) in sorted(per_kernel.items(), key=lambda x: -x[1][1]):
            if t / tot < 0.001:
                continue
            short = name.split("(")[0].replace("void ", "")[:90]
            f.write(f"| `{short}` | {n} | {t / 1e3:.2f} | {100 * t / tot:.1f}% |\n")


def run_e2e_ours(eng, args, B, S, V, dev, rank):
    import torch
    K = args.e2e_steps or args.steps
    host = synthetic_batches(2, B, S, V, None, seed=99 + rank, pinned=True)
    losses = []

    def one(i):
        ids = host[i % len(host)].to(dev, non_blocking=True)
        out = eng.train_step([{"input_ids": ids, "labels": ids}])
        stats = torch.stack([out["loss"], out["grad_norm"]]).cpu()
        losses.append(float(stats[0]))

    for i in range(2):
        one(i)
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(K):
        one(i)
    torch.cuda.synchronize()
    dt = max_over_ranks((time.perf_counter() - t0) / K)
    return {"s_per_step": dt, "h2d": B * S * 8, "d2h": 8,
            "last_loss": losses[-1]}


# -------------------------------------------------------- reference arm
def run_reference(args, world, rank, local):
    import torch
    import torch.nn as nn
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "model")):
        raise FileNotFoundError("baseline/_ref is missing")
    sys.path.insert(0, ref)
    from model.config import ModelConfig as RC  # noqa: E402  (reference code)
    from model.transformer import Qwen3Model as RM
    from training.optimizer import build_optimizer
    from training.scheduler import build_scheduler

    mk, B, S, par = CONFIGS[args.config]
    if DEVICE == "cpu":
        return run_reference_cpu(args, mk, B, S)
    if par == "tp":
        # substituted baseline (the reference's TP path does not run): FSDP2 over the
        # same global batch, i.e. B / N sequences per rank
        B = max(1, B // world)
    rk = dict(mk)
    torch.manual_seed(0)
    model = RM(RC(**rk))
    dev = torch.device("cuda", local)
    model = model.to(dev)
    if world > 1:
        from distributed.parallel import ParallelConfig, ParallelismManager
        pm = ParallelismManager(ParallelConfig(dp_size=-1, fsdp_enabled=True, dtype="bfloat16"))
        model = pm.apply_parallelism(model)
    opt = build_optimizer(model, lr=3e-4, weight_decay=0.1, fused=True)
    sched = build_scheduler(opt, scheduler_type="cosine", warmup_steps=100, total_steps=100000)
    inputs = synthetic_batches(4, B, S, mk["vocab_size"], dev, seed=1234 + rank)

    def step(ids):
        opt.zero_grad()
        with torch.amp.autocast("cuda", dtype=torch.bfloat16):
            out = model(input_ids=ids, labels=ids)
            loss = out["loss"]
        loss.backward()
        loss.item()  # the reference loop reads the loss every micro-step
        nn.utils.clip_grad_norm_(model.parameters(), 1.0)
        opt.step()
        sched.step()

    ms, clocks = timed_loop(step, inputs, args.steps, args.warmup, local)
    e2e = None
    if not args.no_e2e:
        host = synthetic_batches(2, B, S, mk["vocab_size"], None, seed=99 + rank, pinned=True)
        for i in range(2):
            step(host[i].to(dev, non_blocking=True))
        barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        K = args.e2e_steps or args.steps
        for i in range(K):
            ids = host[i % 2].to(dev, non_blocking=True)
            opt.zero_grad()
            with torch.amp.autocast("cuda", dtype=torch.bfloat16):
                out = model(input_ids=ids, labels=ids)
                loss = out["loss"]
            loss.backward()
            gn = nn.utils.clip_grad_norm_(model.parameters(), 1.0)
            opt.step()
            sched.step()
            torch.stack([loss.detach().float(), gn.float() if torch.is_tensor(gn) else loss.detach().float()]).cpu()
        torch.cuda.synchronize()
        e2e = {"s_per_step": max_over_ranks((time.perf_counter() - t0) / K), "h2d": B * S * 8, "d2h": 8}
    return ms, clocks, {}, e2e


def run_reference_cpu(args, mk, B, S):
    """The CPU debug step: the reference's Qwen3Model + build_optimizer (unfused
    AdamW on the CPU) + clip_grad_norm_, fp32, one process, host-timed."""
    import torch
    import torch.nn as nn
    from model.config import ModelConfig as RC  # noqa: E402  (reference code)
    from model.transformer import Qwen3Model as RM
    from training.optimizer import build_optimizer
    torch.manual_seed(0)
    model = RM(RC(**mk))
    opt = build_optimizer(model, lr=3e-4, weight_decay=0.1, fused=False)
    inputs = synthetic_batches(4, B, S, mk["vocab_size"], None, seed=1234)

    def step(ids):
        opt.zero_grad()
        out = model(input_ids=ids, labels=ids)
        out["loss"].backward()
        nn.utils.clip_grad_norm_(model.parameters(), 1.0)
        opt.step()

    ms, clocks = timed_loop(step, inputs, args.steps, args.warmup, 0)
    return ms, clocks, {}, None


def parallel_label(par, world, impl, mode):
    if world == 1:
        return "dp1"
    if impl == "reference":
        return f"dp{world} (FSDP2{', substituted for the reference TP/EP paths, which do not run' if par != 'dp' else ''})"
    if par == "tp":
        return f"tp{world}+sp (" + ("all-gather / reduce-scatter fused into the norm and GEMM kernels over peer memory"
                                    if mode == "tp-fused" else "NCCL collectives") + ")"
    if par == "cp":
        if mode == "cp-ring":
            return f"cp{world} (zigzag; k|v ring over NCCL send/recv, flash kernels per chunk pair)"
        return f"cp{world} (zigzag; K/V exchange by P2P stores consumed by the attention kernels)"
    if par == "ep":
        return f"ep{world} x dp{world} (" + ("dispatch/combine kernels over peer memory" if mode == "ep-fused"
                                             else "NCCL all-to-all dispatch/combine") + ")"
    return f"dp{world} ({DP_LABEL.get(mode, '')})"


# --------------------------------------------------------------------- main
def main():
    args = parse()
    import torch
    global DEVICE
    DEVICE = args.device
    world, rank, local = dist_setup()
    if DEVICE == "cpu" and world > 1:
        print(json.dumps({"error": "--device cpu runs one process"}))
        return 2
    if args.gpus != world and world == 1 and args.gpus > 1:
        print(json.dumps({"error": "launch N>1 with torch.distributed.run"}))
        return 2
    mk, B, S, par = CONFIGS[args.config]
    global KERNEL_TABLE
    KERNEL_TABLE = args.kernel_table if rank == 0 else None
    if args.impl == "reference" and par == "cp" and world > 1:
        maybe_init_pg(world, local)
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "the reference never wires context "
                              "parallelism (RingAttention is unused, distributed/context_parallel.py)"}))
        return 0
    try:
        if args.impl == "reference":
            maybe_init_pg(world, local)
            ms, clocks, extra, e2e = run_reference(args, world, rank, local)
        else:
            ms, clocks, extra, e2e = run_ours(args, world, rank, local)
    except FileNotFoundError as e:
        if rank == 0:
            print(json.dumps({"impl": args.impl, "unavailable": str(e)}))
        return 0
    tokens_per_step = B * S * (1 if par in ("tp", "cp") else world)
    value = tokens_per_step / (ms / 1e3)
    fpt = flops_per_token(mk, S)
    mfu = value * fpt / (measured_peak() * world) if DEVICE == "cuda" else None
    line = {
        "metric": BASELINE_METRIC,
        "value": round(value, 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 3),
        "higher_is_better": True,
        "scaling": "strong" if par in ("tp", "cp") else "weak",
        "vs_baseline": (round(value / CPU_BASELINE_TOKS, 3)
                        if DEVICE == "cpu" and args.config == "debug" else None),
        "dtype": "bf16" if DEVICE == "cuda" else "fp32",
        "data": "synthetic uniform-random token ids, random-init weights",
        "config": {"model": f"{args.config} (Qwen3-1.7B shape: L28 h2048 16Q/8KV hd128 I6144 V151936 tied)"
                   if args.config == "qwen3-1.7b" else args.config,
                   "global_batch": B * (1 if par in ("tp", "cp") else world), "seq_len": S,
                   "parallelism": parallel_label(par, world, args.impl, extra.get("dp_mode")),
                   "l2": "no flush: per-step working set (weights + activations) >> 126 MB L2"},
        "mfu": round(mfu, 4) if mfu is not None else None,
        "flops_per_token": fpt,
        "clocks": clocks,
    }
    if args.impl == "reference":
        line["impl"] = "reference"
    else:
        line["impl"] = "ours"
        line["gpu_launches"] = extra["gpu_launches_per_step"]["ours"] * args.steps
        line["launches_per_step"] = extra["gpu_launches_per_step"]
        line["kernel_error_flag"] = extra["kernel_error_flag"]
        # the data-parallel optimizer step that ran: p2p (peer memory),
        # shard (NCCL ZeRO-2), replicate, fsdp, or none (one replica)
        line["dp_step"] = extra.get("dp_step")
    if e2e is not None:
        line["e2e"] = {"value": round(tokens_per_step / e2e["s_per_step"], 1), "unit": "tokens/s",
                       "h2d_bytes_per_step": e2e["h2d"], "d2h_bytes_per_step": e2e["d2h"]}
    if rank == 0:
        print(json.dumps(line), flush=True)
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
