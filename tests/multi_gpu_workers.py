"""Worker functions for tests that need two or more GPUs (NCCL, one process
per GPU, spawned by ``test_multi_gpu.py``)."""

from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist


def init(rank: int, world: int, port: int) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))


def _cfg():
    from nano_qwen_b200.config import ModelConfig
    return ModelConfig(hidden_size=256, num_hidden_layers=2, num_attention_heads=4,
                       num_key_value_heads=2, head_dim=64, intermediate_size=512,
                       vocab_size=4096, max_position_embeddings=512, tie_word_embeddings=True)


def _engine(mode, group, overlap=False):
    from nano_qwen_b200.models import Qwen3Model
    from nano_qwen_b200.training.engine import TrainEngine
    torch.manual_seed(0)
    dev = torch.device("cuda", torch.cuda.current_device())
    tc = {"optimizer": {"lr": 1e-3, "grad_clip": 0.5},
          "scheduler": {"warmup_steps": 0, "total_steps": 10},
          "distributed": {"overlap_grad_reduce": overlap}}
    return TrainEngine(Qwen3Model(_cfg()), tc, dev, dp_mode=mode, dp_group=group)


def peer_dp_worker(rank, world, port):
    """The peer-memory fused ZeRO step equals single-process gradient
    accumulation over every rank's micro-batch, and the NCCL ZeRO-2 path."""
    init(rank, world, port)
    from nano_qwen_b200.ops import ext
    singles = [dist.new_group([r]) for r in range(world)]
    g = torch.Generator().manual_seed(5)
    ids = torch.randint(0, 4096, (2 * world, 128), generator=g).cuda()
    mine = [{"input_ids": ids[2 * rank:2 * rank + 2], "labels": ids[2 * rank:2 * rank + 2]}]
    full = [{"input_ids": ids[i:i + 2], "labels": ids[i:i + 2]} for i in range(0, 2 * world, 2)]
    ref = _engine(None, singles[rank])
    p2p = _engine("p2p", None)
    assert hasattr(p2p.dp, "fused_step"), "symmetric memory unavailable"
    nccl = _engine("shard", None)
    ovl = _engine("p2p", None, overlap=True)  # per-block reduce-scatter during the backward
    novl = _engine("shard", None, overlap=True)  # the same with NCCL on a side stream
    log = []
    for _ in range(3):
        r = ref.train_step(full)
        a = p2p.train_step(mine)
        b = nccl.train_step(mine)
        c = ovl.train_step(mine)
        d = novl.train_step(mine)
        assert novl.dp.last_overlapped == len(novl.dp._hooked) > 0
        log.append([float(x[k]) for x in (r, a, b, c, d) for k in ("loss", "grad_norm")])
    torch.cuda.synchronize()
    assert ext().error_flag_read() == 0, "kernel error word set"
    for x in (a, b, c, d):
        assert abs(float(x["grad_norm"]) - float(r["grad_norm"])) < 1e-3 * float(r["grad_norm"]), \
            f"rank {rank} (loss, norm) ref/p2p/nccl per step: {log}"
    p2p.state_for_save()
    ovl.state_for_save()
    nccl.state_for_save()
    novl.state_for_save()
    def rel(a_, b_):
        return ((a_ - b_).norm() / (b_.norm() + 1e-12)).item()

    for (n, p), q, s, o, no in zip(ref.model.named_parameters(), p2p.model.parameters(),
                                   nccl.model.parameters(), ovl.model.parameters(),
                                   novl.model.parameters()):
        # the data-parallel paths reduce the same per-rank gradients
        assert rel(q, s) < 1e-3, (n, rel(q, s))
        assert rel(q, o) < 1e-3, (n, rel(q, o))
        assert rel(s, no) < 1e-3, (n, rel(s, no))
        # against gradient accumulation in one process the fp32 summation order
        # differs, and Adam's m/sqrt(v) amplifies that on near-zero gradients
        assert rel(q, p) < 2e-3, (n, rel(q, p))
    # every rank's bf16 compute copy holds the same (all-gathered) weights
    comp = p2p.store.compute.float()
    tot = comp.clone()
    dist.all_reduce(tot)
    assert torch.equal(tot, comp * world)
    dist.barrier()
    del p2p
    dist.destroy_process_group()


def tp_fused_worker(rank, world, port):
    """Fused TP+SP (collectives inside the norm and GEMM kernels) against the
    single-GPU model and against the NCCL TP+SP path: loss and gradients."""
    init(rank, world, port)
    from nano_qwen_b200.models import Qwen3Model
    from nano_qwen_b200.ops import ext
    from nano_qwen_b200.parallel.tensor_parallel import apply_tensor_parallel, sync_replicated_grads
    from nano_qwen_b200.training.optimizer import attach_param_store
    from nano_qwen_b200.config import ModelConfig
    # 16 Q / 8 KV heads divide by every tp size up to 8; 2 x 512 tokens give
    # each rank a multiple of 128 rows under sequence parallelism
    cfg = ModelConfig(hidden_size=256, num_hidden_layers=2, num_attention_heads=16,
                      num_key_value_heads=8, head_dim=64, intermediate_size=1024,
                      vocab_size=4096, max_position_embeddings=1024, tie_word_embeddings=True)
    grp = dist.new_group(list(range(world)))
    g = torch.Generator().manual_seed(7)
    ids = torch.randint(0, cfg.vocab_size, (2, 512), generator=g).cuda()

    def build(tp, fused):
        torch.manual_seed(0)
        m = Qwen3Model(cfg).cuda()
        with torch.no_grad():
            for n, p in m.named_parameters():
                if p.ndim >= 2:
                    p.normal_(0.0, 0.05)
        if tp:
            apply_tensor_parallel(m, grp, sequence_parallel=True, fused=fused)
        attach_param_store(m)
        return m

    def run(m, tp):
        out = m(ids, labels=ids)
        out["loss"].backward()
        if tp:
            sync_replicated_grads(m, grp)
        torch.cuda.synchronize()
        return out["loss"].detach().float()

    ref = build(False, False)
    l_ref = run(ref, False)
    fused = build(True, True)
    assert getattr(fused, "tp_fused", False), "fused TP path not enabled"
    l_fused = run(fused, True)
    nccl = build(True, False)
    l_nccl = run(nccl, True)
    assert ext().error_flag_read() == 0, "kernel error word set"
    assert abs(float(l_fused) - float(l_ref)) < 1e-2 * float(l_ref), (float(l_fused), float(l_ref))
    assert abs(float(l_fused) - float(l_nccl)) < 5e-3 * float(l_ref), (float(l_fused), float(l_nccl))
    rp = dict(ref.named_parameters())
    worst = {}
    for (n, p), q in zip(fused.named_parameters(), nccl.parameters()):
        g_ref = rp[n].grad
        if getattr(p, "_tp_sharded", False):
            if p.shape[0] != g_ref.shape[0]:
                k = p.shape[0]
                g_ref = g_ref[rank * k:(rank + 1) * k]
            else:
                k = p.shape[1]
                g_ref = g_ref[:, rank * k:(rank + 1) * k]
        e1 = ((p.grad.float() - g_ref.float()).norm() / (g_ref.float().norm() + 1e-12)).item()
        e2 = ((p.grad.float() - q.grad.float()).norm() / (q.grad.float().norm() + 1e-12)).item()
        worst[n] = (round(e1, 4), round(e2, 4))
        assert e1 < 0.05 and e2 < 0.05, (n, e1, e2, worst)
    dist.barrier()
    dist.destroy_process_group()


def ep_fused_worker(rank, world, port):
    """Fused expert parallelism (peer-memory dispatch/combine kernels) against
    the single-GPU MoE layer: loss on this rank's tokens, dense gradients, and
    expert gradients summed over the ranks' tokens."""
    init(rank, world, port)
    from nano_qwen_b200.config import ModelConfig
    from nano_qwen_b200.models import Qwen3Model
    from nano_qwen_b200.ops import ext
    from nano_qwen_b200.parallel.expert_parallel import apply_expert_parallel
    from nano_qwen_b200.training.optimizer import attach_param_store
    cfg = ModelConfig(hidden_size=256, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=64, intermediate_size=512, vocab_size=4096,
                      max_position_embeddings=512, tie_word_embeddings=True, num_experts=8,
                      num_experts_per_tok=2, moe_intermediate_size=128)
    grp = dist.new_group(list(range(world)))
    g = torch.Generator().manual_seed(11 + rank)
    ids = torch.randint(0, cfg.vocab_size, (2, 256), generator=g).cuda()

    def build(ep, fused):
        torch.manual_seed(0)
        m = Qwen3Model(cfg).cuda()
        with torch.no_grad():
            for n, p in m.named_parameters():
                if p.ndim >= 2:
                    p.normal_(0.0, 0.05)
        if ep:
            apply_expert_parallel(m, grp, fused=fused)
        attach_param_store(m)
        return m

    ref = build(False, False)
    out = ref(ids, labels=ids)
    out["loss"].backward()
    l_ref = float(out["loss"])
    ref_g = {n: p.grad.float().clone() for n, p in ref.named_parameters()}
    for n in ref_g:
        if ".experts." in n:
            dist.all_reduce(ref_g[n], group=grp)  # owner's expert grad covers every rank's tokens
    results = {}
    for fused in (True, False):
        m = build(True, fused)
        o = m(ids, labels=ids)
        o["loss"].backward()
        torch.cuda.synchronize()
        results[fused] = (float(o["loss"]), {n: p.grad.float() for n, p in m.named_parameters()})
    assert ext().error_flag_read() == 0, "kernel error word set"
    e_loc = cfg.num_experts // world
    for fused, (loss, grads) in results.items():
        assert abs(loss - l_ref) < 2e-3 * l_ref, (fused, loss, l_ref)
        for n, gr in grads.items():
            rn = n
            if ".experts." in n:
                pre, rest = n.split(".experts.", 1)
                e, tail = rest.split(".", 1)
                rn = f"{pre}.experts.{int(e) + rank * e_loc}.{tail}"
            err = ((gr - ref_g[rn]).norm() / (ref_g[rn].norm() + 1e-12)).item()
            assert err < 2e-2, (fused, n, err)
    # global-batch load balancing: the fused path takes the counts from its
    # own exchange, the NCCL path all-reduces them; both give the same loss
    from nano_qwen_b200.training.engine import set_global_batch_balance
    aux = {}
    for fused in (True, False):
        m = build(True, fused)
        set_global_batch_balance(m, grp)
        o = m(ids, labels=ids)
        o["loss"].backward()
        torch.cuda.synchronize()
        aux[fused] = (float(o["loss"]), float(o["aux_loss"]))
    assert ext().error_flag_read() == 0
    assert abs(aux[True][1] - aux[False][1]) < 1e-4 * abs(aux[False][1]), aux
    assert abs(aux[True][0] - aux[False][0]) < 2e-3 * aux[False][0], aux
    dist.barrier()
    dist.destroy_process_group()


def cp_kernel_worker(rank, world, port, mode="allgather"):
    """Context parallelism on the attention kernels (zigzag over the ranks) against
    the single-GPU model on the full sequence: loss and gradients.  ``mode``:
    gathered k|v (peer-memory kernels) or the k|v ring."""
    init(rank, world, port)
    from nano_qwen_b200.models import Qwen3Model
    from nano_qwen_b200.ops import ext
    from nano_qwen_b200.parallel.context_parallel import apply_context_parallel
    from nano_qwen_b200.training.optimizer import attach_param_store
    from nano_qwen_b200.config import ModelConfig
    cfg = ModelConfig(hidden_size=256, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                      head_dim=128, intermediate_size=512, vocab_size=4096,
                      max_position_embeddings=2048, tie_word_embeddings=True)
    grp = dist.new_group(list(range(world)))
    g = torch.Generator().manual_seed(3)
    ids = torch.randint(0, cfg.vocab_size, (1, 2048), generator=g).cuda()

    def build(cp):
        torch.manual_seed(0)
        m = Qwen3Model(cfg).cuda()
        with torch.no_grad():
            for n, p in m.named_parameters():
                if p.ndim >= 2:
                    p.normal_(0.0, 0.05)
        if cp:
            apply_context_parallel(m, grp, mode=mode)
        attach_param_store(m)
        return m

    ref = build(False)
    o = ref(ids, labels=ids)
    o["loss"].backward()
    cpm = build(True)
    oc = cpm(ids, labels=ids)
    oc["loss"].backward()
    torch.cuda.synchronize()
    assert ext().error_flag_read() == 0, "kernel error word set"
    lc, lr = float(oc["loss"].detach()), float(o["loss"].detach())
    assert abs(lc - lr) < 1e-2 * lr, (lc, lr)
    rp = dict(ref.named_parameters())
    for n, p in cpm.named_parameters():
        gsum = p.grad.float().clone()
        # the CP loss back-propagates cp x the rank's partial gradient, so the
        # data-parallel average over the group is the full-sequence gradient
        dist.all_reduce(gsum, group=grp)
        gsum /= world
        gr = rp[n].grad.float()
        err = ((gsum - gr).norm() / (gr.norm() + 1e-12)).item()
        assert err < 5e-2, (n, err)
    dist.barrier()
    dist.destroy_process_group()


def fsdp_worker(rank, world, port):
    """Fully sharded parameters over NCCL (per-block bf16 all-gathers with
    prefetch, fp32 reduce-scatters on a side stream) against the NCCL ZeRO-2
    step on the same ranks and data: losses, norms and final weights."""
    init(rank, world, port)
    from nano_qwen_b200.ops import ext
    from nano_qwen_b200.parallel.fsdp import _FREE
    g = torch.Generator().manual_seed(5)
    ids = torch.randint(0, 4096, (4 * world, 128), generator=g).cuda()
    mine = [{"input_ids": ids[4 * rank + i:4 * rank + i + 2],
             "labels": ids[4 * rank + i:4 * rank + i + 2]} for i in (0, 2)]
    zero = _engine("shard", None)
    fs = _engine("fsdp", None)
    assert fs.store.mode == "fsdp" and fs.store.nccl
    total = sum(p.numel() for p in zero.model.parameters())
    assert fs.store.master.numel() < total // world + 64 * len(fs.store.units)
    for _ in range(3):
        a = zero.train_step(mine)
        b = fs.train_step(mine)
        assert abs(float(a["loss"]) - float(b["loss"])) < 1e-4 * abs(float(a["loss"])), (a, b)
        assert abs(float(a["grad_norm"]) - float(b["grad_norm"])) < 1e-3 * float(a["grad_norm"])
        assert all(u.state == _FREE for u in fs.store.block_units[:-1])
    torch.cuda.synchronize()
    assert ext().error_flag_read() == 0, "kernel error word set"
    zero.state_for_save()
    fs.state_for_save()
    for (n, p), q in zip(zero.model.named_parameters(), fs.model.parameters()):
        err = ((p - q).norm() / (p.norm() + 1e-12)).item()
        assert err < 1e-3, (n, err)
    fs.optimizer.release_full_state()
    dist.barrier()
    dist.destroy_process_group()


def rank_leave_worker(rank, world, port):
    """One process per GPU trains with NCCL data parallelism; the last rank
    leaves between steps (synchronised, then exits without a word).  The
    survivors' host-side step gate names it before they launch their next
    collective.  NVLS is off and no buffer is bound to a multicast object, so
    the departed rank's memory is not part of anything the survivors touch."""
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["TORCH_SYMM_MEM_DISABLE_MULTICAST"] = "1"
    init(rank, world, port)
    from nano_qwen_b200.ops import ext
    from nano_qwen_b200.utils.fault import HeartbeatMonitor, PeerFailure
    store = dist.distributed_c10d._get_default_store()
    # generous: the first steps of live ranks can drift apart by seconds
    hb = HeartbeatMonitor(store, rank, world, timeout_s=10.0, prefix="leave")
    eng = _engine("shard", None)  # NCCL reduce-scatter / all-gather, no peer-memory kernels
    g = torch.Generator().manual_seed(21 + rank)
    ids = torch.randint(0, 4096, (2, 128), generator=g).cuda()
    leaver = world - 1
    for step in range(4):
        if rank == leaver and step == 2:
            torch.cuda.synchronize()  # nothing of this rank in flight
            os._exit(0)
        try:
            hb.gate(step)
        except PeerFailure as e:
            assert rank != leaver and step == 2 and e.ranks == [leaver], (rank, step, e.ranks)
            torch.cuda.synchronize()
            assert ext().error_flag_read() == 0
            store.set(f"leave/seen/{rank}", "1")
            if rank == 0:  # hosts the store: leaves after the other survivors
                store.wait([f"leave/seen/{r}" for r in range(1, leaver)], datetime.timedelta(seconds=30))
            os._exit(0)
        out = eng.train_step([{"input_ids": ids, "labels": ids}])
        assert torch.isfinite(out["loss"]).item()
    raise AssertionError("the departed rank was not detected")


def pp_worker(rank, world, port):
    """Pipeline parallelism over NCCL on GPUs (1F1B, micro-batches, tied
    embeddings across the first and last stage) against the single-GPU model."""
    init(rank, world, port)
    from nano_qwen_b200.config import ModelConfig
    from nano_qwen_b200.models import Qwen3Model
    from nano_qwen_b200.ops import ext
    from nano_qwen_b200.parallel.pipeline_parallel import apply_pipeline_parallel
    from nano_qwen_b200.training.optimizer import attach_param_store
    cfg = ModelConfig(hidden_size=256, num_hidden_layers=2 * world, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=64, intermediate_size=512, vocab_size=4096,
                      max_position_embeddings=512, tie_word_embeddings=True)
    g = torch.Generator().manual_seed(13)
    ids = torch.randint(0, cfg.vocab_size, (4, 256), generator=g).cuda()

    def build():
        torch.manual_seed(0)
        m = Qwen3Model(cfg).cuda()
        with torch.no_grad():
            for p in m.parameters():
                if p.ndim >= 2:
                    p.normal_(0.0, 0.05)
        return m

    ref = build()
    attach_param_store(ref)
    loss_ref = 0.0
    for c in ids.chunk(4):
        o = ref(c, labels=c)
        (o["loss"] / 4).backward()
        loss_ref += float(o["loss"]) / 4
    grp = dist.new_group(list(range(world)))
    pm = apply_pipeline_parallel(build(), grp, list(range(world)), n_microbatches=4)
    attach_param_store(pm.model)
    loss, _ = pm.pipeline_forward_backward([{"input_ids": ids, "labels": ids}])
    torch.cuda.synchronize()
    assert ext().error_flag_read() == 0
    assert abs(float(loss) - loss_ref) < 1e-2 * loss_ref, (float(loss), loss_ref)
    rp = dict(ref.named_parameters())
    off = pm.stage_layers[rank][0]
    for n, p in pm.model.named_parameters():
        rn = n
        if n.startswith("layers."):
            i, tail = n[len("layers."):].split(".", 1)
            rn = f"layers.{int(i) + off}.{tail}"
        if rn == "lm_head.weight":
            rn = "embed.embed_tokens.weight"
        gr = rp[rn].grad.float()
        err = ((p.grad.float() - gr).norm() / (gr.norm() + 1e-12)).item()
        assert err < 5e-2, (n, err)
    dist.barrier()
    dist.destroy_process_group()


def peer_dp_layout_worker(rank, world, port):
    """The peer-memory data-parallel step under model-parallel layouts
    (``dp_mode="p2p"`` with a ``ParallelismManager``): expert parallelism
    (the expert span reduced over the ranks holding the same experts) and
    tensor parallelism, against the NCCL ZeRO step on the same layout, three
    steps: losses, gradient norms, then every weight."""
    init(rank, world, port)
    from nano_qwen_b200.config import ModelConfig
    from nano_qwen_b200.models import Qwen3Model
    from nano_qwen_b200.ops import ext
    from nano_qwen_b200.parallel.manager import ParallelConfig, ParallelismManager
    from nano_qwen_b200.parallel.peer_dp import PeerDataParallel
    from nano_qwen_b200.training.engine import TrainEngine
    cfg = ModelConfig(hidden_size=256, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=64, intermediate_size=512, vocab_size=4096,
                      max_position_embeddings=512, tie_word_embeddings=True, num_experts=8,
                      num_experts_per_tok=2, moe_intermediate_size=128)
    dev = torch.device("cuda", rank)
    tc = {"optimizer": {"lr": 1e-3, "grad_clip": 0.5},
          "scheduler": {"warmup_steps": 0, "total_steps": 10}}
    layouts = [{"ep_size": 2}] + ([{"tp_size": 2}] if world >= 4 else [])
    for layout in layouts:
        engines = {}
        for mode in ("p2p", "shard"):
            torch.manual_seed(0)
            pm = ParallelismManager(ParallelConfig(**layout))
            m = Qwen3Model(cfg).to(dev)
            engines[mode] = (TrainEngine(pm.apply_parallelism(m), tc, dev, dp_mode=mode, parallel=pm), pm)
        p2p, pm = engines["p2p"]
        nccl, _ = engines["shard"]
        assert isinstance(p2p.dp, PeerDataParallel), "symmetric memory unavailable"
        d = pm.coords["dp"]
        g = torch.Generator().manual_seed(21)
        for step in range(3):
            ids = torch.randint(0, cfg.vocab_size, (2 * pm.config.dp_size, 128), generator=g).to(dev)
            mb = [{"input_ids": ids[2 * d:2 * d + 2], "labels": ids[2 * d:2 * d + 2]}]
            a = p2p.train_step(mb)
            b = nccl.train_step(mb)
            assert abs(float(a["loss"]) - float(b["loss"])) < 2e-3 * float(b["loss"]), (layout, step)
            assert abs(float(a["grad_norm"]) - float(b["grad_norm"])) < 2e-3 * float(b["grad_norm"]), \
                (layout, step, float(a["grad_norm"]), float(b["grad_norm"]))
        torch.cuda.synchronize()
        assert ext().error_flag_read() == 0, "kernel error word set"
        p2p.state_for_save()
        nccl.state_for_save()
        for (n, q), s in zip(p2p.model.named_parameters(), nccl.model.parameters()):
            err = ((q.float() - s.float()).norm() / (s.float().norm() + 1e-12)).item()
            assert err < 2e-3, (layout, n, err)
        dist.barrier()
        del p2p, nccl, engines
    dist.destroy_process_group()
