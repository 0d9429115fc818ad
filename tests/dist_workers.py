"""Worker functions for the multi-rank CPU tests (Gloo, spawned processes).

Every worker builds the same tiny model from the same seed, computes a
single-process oracle locally (the full model on the full batch), runs the
parallel variant and asserts agreement; an assertion error in any rank fails
the spawning test.
"""

from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist


def init(rank: int, world: int, port: int) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["RANK"] = str(rank)
    os.environ["WORLD_SIZE"] = str(world)
    os.environ["LOCAL_RANK"] = str(rank)
    torch.set_num_threads(1)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))


def tiny_cfg(moe: bool = False, **kw):
    from nano_qwen_b200.config import ModelConfig
    base = dict(hidden_size=32, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                head_dim=8, intermediate_size=64, vocab_size=97, max_position_embeddings=64,
                tie_word_embeddings=False, rope_theta=1e4)
    if moe:
        base.update(num_experts=4, num_experts_per_tok=2, moe_intermediate_size=16)
    base.update(kw)
    return ModelConfig(**base)


def build(cfg, seed: int = 0):
    from nano_qwen_b200.models import Qwen3Model
    torch.manual_seed(seed)
    m = Qwen3Model(cfg)
    with torch.no_grad():  # larger than the default init so the test sees real gradients
        for n, p in m.named_parameters():
            if p.ndim >= 2:
                p.normal_(0.0, 0.2)
    return m


def batch(cfg, B: int, S: int, seed: int = 1):
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, cfg.vocab_size, (B, S), generator=g)
    return ids


def close(a, b, tol=2e-4, what=""):
    a, b = a.detach().float(), b.detach().float()
    err = ((a - b).norm() / (b.norm() + 1e-8)).item()
    assert err < tol, f"{what}: rel err {err:.3e}"


def _full_grads(cfg, ids, moe_scale=False):
    ref = build(cfg)
    out = ref(ids, labels=ids)
    out["loss"].backward()
    return ref, out["loss"].detach(), {n: p.grad.clone() for n, p in ref.named_parameters()}


# ------------------------------------------------------------------ TP (+SP)
def tp_worker(rank, world, port, sp, moe):
    init(rank, world, port)
    from nano_qwen_b200.parallel.tensor_parallel import apply_tensor_parallel, sync_replicated_grads
    cfg = tiny_cfg(moe)
    ids = batch(cfg, 2, 16)
    ref, ref_loss, ref_g = _full_grads(cfg, ids)
    m = build(cfg)
    grp = dist.new_group(list(range(world)))
    apply_tensor_parallel(m, grp, sequence_parallel=sp)
    out = m(ids, labels=ids)
    out["loss"].backward()
    sync_replicated_grads(m, grp)
    close(out["loss"], ref_loss, 1e-5, "loss")
    for n, p in m.named_parameters():
        g = ref_g[n]
        if getattr(p, "_tp_sharded", False):
            if p.shape[0] != g.shape[0]:  # row shard (column-parallel)
                k = p.shape[0]
                g = g[rank * k:(rank + 1) * k]
            else:                         # column shard (row-parallel)
                k = p.shape[1]
                g = g[:, rank * k:(rank + 1) * k]
        close(p.grad, g, 2e-4, n)
    dist.destroy_process_group()


# ------------------------------------------------------------------ DP
def dp_worker(rank, world, port, mode):
    init(rank, world, port)
    from nano_qwen_b200.training.engine import TrainEngine
    cfg = tiny_cfg()
    ids = batch(cfg, 2 * world, 16)
    tcfg = {"optimizer": {"lr": 1e-2, "grad_clip": 1.0},
            "scheduler": {"warmup_steps": 0, "total_steps": 10}}
    ref = TrainEngine(build(cfg), tcfg, torch.device("cpu"))
    full = [{"input_ids": ids[i:i + 2], "labels": ids[i:i + 2]} for i in range(0, 2 * world, 2)]
    for _ in range(2):
        r_out = ref.train_step(full)
    eng = TrainEngine(build(cfg), tcfg, torch.device("cpu"), dp_mode=mode)
    mine = [{"input_ids": ids[2 * rank:2 * rank + 2], "labels": ids[2 * rank:2 * rank + 2]}]
    for _ in range(2):
        o = eng.train_step(mine)
    eng.state_for_save()
    close(o["grad_norm"], r_out["grad_norm"], 1e-4, "grad norm")
    for (n, p), (_, q) in zip(eng.model.named_parameters(), ref.model.named_parameters()):
        close(p, q, 1e-5, n)
    dist.destroy_process_group()


# ------------------------------------------------------------------ EP
def ep_worker(rank, world, port):
    init(rank, world, port)
    from nano_qwen_b200.parallel.data_parallel import DataParallel
    from nano_qwen_b200.parallel.expert_parallel import apply_expert_parallel
    from nano_qwen_b200.training.optimizer import attach_param_store
    cfg = tiny_cfg(moe=True)
    ids = batch(cfg, 2 * world, 16)
    # oracle: mean of the per-rank losses = loss over all micro-batches
    ref = build(cfg)
    ref_losses = []
    for r in range(world):
        o = ref(ids[2 * r:2 * r + 2], labels=ids[2 * r:2 * r + 2])
        (o["loss"] / world).backward()
        ref_losses.append(o["loss"].detach())
    ref_g = {n: p.grad.clone() for n, p in ref.named_parameters()}
    m = build(cfg)
    grp = dist.new_group(list(range(world)))
    apply_expert_parallel(m, grp)
    store = attach_param_store(m, torch.float32, torch.device("cpu"))
    dp = DataParallel(store, mode="replicate", group=grp, expert_group=None)
    out = m(ids[2 * rank:2 * rank + 2], labels=ids[2 * rank:2 * rank + 2])
    out["loss"].backward()
    close(out["loss"], ref_losses[rank], 1e-5, "loss")
    dp.sync_grads()
    e_loc = cfg.num_experts // world
    for n, p in m.named_parameters():
        rn = n
        if ".experts." in n:
            pre, rest = n.split(".experts.", 1)
            e, tail = rest.split(".", 1)
            rn = f"{pre}.experts.{int(e) + rank * e_loc}.{tail}"
        close(p.grad, ref_g[rn], 2e-4, n)
    dist.destroy_process_group()


# ------------------------------------------------------------------ CP
def cp_worker(rank, world, port, moe, mode="allgather"):
    init(rank, world, port)
    from nano_qwen_b200.parallel.context_parallel import apply_context_parallel
    from nano_qwen_b200.parallel.data_parallel import DataParallel
    from nano_qwen_b200.training.optimizer import attach_param_store
    # aux-loss statistics are per rank under CP, so the exact comparison runs with coef 0
    cfg = tiny_cfg(moe, router_aux_loss_coef=0.0)
    ids = batch(cfg, 2, 8 * world)
    ref, ref_loss, ref_g = _full_grads(cfg, ids)
    m = build(cfg)
    grp = dist.new_group(list(range(world)))
    apply_context_parallel(m, grp, mode=mode)
    store = attach_param_store(m, torch.float32, torch.device("cpu"))
    dp = DataParallel(store, mode="replicate", group=grp)
    out = m(ids, labels=ids)
    out["loss"].backward()
    dp.sync_grads()
    close(out["loss"], ref_loss, 1e-5, "loss")
    for n, p in m.named_parameters():
        close(p.grad, ref_g[n], 2e-4, n)
    logits = m(ids)["logits"]
    close(logits, ref(ids)["logits"], 1e-5, "logits")
    dist.destroy_process_group()


# ------------------------------------------------------------------ PP
def pp_worker(rank, world, port, tied, micro):
    init(rank, world, port)
    from nano_qwen_b200.parallel.pipeline_parallel import apply_pipeline_parallel
    cfg = tiny_cfg(tie_word_embeddings=tied, num_hidden_layers=4)
    ids = batch(cfg, 4, 16)
    ref = build(cfg)
    loss_ref = 0.0
    for c in ids.chunk(micro):
        o = ref(c, labels=c)
        (o["loss"] / micro).backward()
        loss_ref += o["loss"].item() / micro
    ref_g = {n: p.grad.clone() for n, p in ref.named_parameters()}
    m = build(cfg)
    grp = dist.new_group(list(range(world)))
    pm = apply_pipeline_parallel(m, grp, list(range(world)), n_microbatches=micro)
    loss, _ = pm.pipeline_forward_backward([{"input_ids": ids, "labels": ids}])
    assert abs(loss.item() - loss_ref) < 1e-5 * max(1.0, abs(loss_ref)), (loss.item(), loss_ref)
    off = pm.stage_layers[rank][0]
    for n, p in pm.model.named_parameters():
        rn = n
        if n.startswith("layers."):
            i, tail = n[len("layers."):].split(".", 1)
            rn = f"layers.{int(i) + off}.{tail}"
        if tied and rn == "lm_head.weight":
            rn = "embed.embed_tokens.weight"
        close(p.grad, ref_g[rn], 2e-4, n)
    dist.destroy_process_group()


# ------------------------------------------------------------------ manager
def manager_worker(rank, world, port, tp, cp, pp, ep):
    init(rank, world, port)
    from nano_qwen_b200.parallel.manager import ParallelConfig, ParallelismManager
    pm = ParallelismManager(ParallelConfig(tp_size=tp, cp_size=cp, pp_size=pp, ep_size=ep))
    c = pm.coords
    assert pm.ranks["tp"] == [r for r in range(world) if r // tp == rank // tp]
    for axis in ("tp", "cp", "dp", "pp"):
        assert rank in pm.ranks[axis]
    assert len(pm.ranks["dp"]) == pm.config.dp_size
    assert len(pm.ranks["ep"]) == ep
    if ep > 1:
        assert len(pm.ranks["edp"]) == pm.config.dp_size // ep
    assert c["tp"] == rank % tp
    dist.destroy_process_group()


# ------------------------------------------------------------------ failure detection
def heartbeat_worker(rank, world, port, dead_rank):
    init(rank, world, port)
    from nano_qwen_b200.utils.fault import HeartbeatMonitor, PeerFailure
    store = dist.distributed_c10d._get_default_store()
    mon = HeartbeatMonitor(store, rank, world, interval_s=0.1, timeout_s=2.0)
    mon.beat()
    if rank == dead_rank:
        return  # leaves between steps without further heartbeats (no collective in flight)
    import time
    t0 = time.time()
    failed = None
    while time.time() - t0 < 10.0:
        mon.beat()
        try:
            mon.check()
        except PeerFailure as e:
            failed = e
            break
        time.sleep(0.1)
    assert failed is not None and dead_rank in failed.ranks, failed


# ------------------------------------------------------------------ checkpoint (model parallel)
def tp_checkpoint_worker(rank, world, port, tmp):
    init(rank, world, port)
    from nano_qwen_b200.parallel.tensor_parallel import apply_tensor_parallel
    from nano_qwen_b200.training.checkpoint import CheckpointManager
    from nano_qwen_b200.training.engine import TrainEngine
    cfg = tiny_cfg()
    ids = batch(cfg, 2, 16)
    grp = dist.new_group(list(range(world)))
    tcfg = {"optimizer": {"lr": 1e-2}, "scheduler": {"warmup_steps": 0, "total_steps": 10}}

    singles = [dist.new_group([r]) for r in range(world)]
    e1 = TrainEngine(apply_tensor_parallel(build(cfg), grp, sequence_parallel=True), tcfg,
                     torch.device("cpu"), dp_group=singles[rank])
    e1.tp_group = grp
    e1.train_step([{"input_ids": ids, "labels": ids}])
    mgr = CheckpointManager(save_dir=tmp, save_interval=1, async_save=False)
    m, o, s = e1.state_for_save()
    path = mgr.save(1, m, o, s, extra_state={"step": 1})
    e2 = TrainEngine(apply_tensor_parallel(build(cfg, seed=5), grp, sequence_parallel=True), tcfg,
                     torch.device("cpu"), dp_group=singles[rank])
    e2.tp_group = grp
    mgr.load(e2.model, e2.optimizer, e2.scheduler, str(path))
    for (n, p), q in zip(e1.model.named_parameters(), e2.model.parameters()):
        assert torch.equal(p, q), n
    # the same checkpoint loads at tp1 (the single-process layout): weights and
    # Adam moments are the concatenation of the tp2 shards
    e3 = TrainEngine(build(cfg, seed=9), tcfg, torch.device("cpu"), dp_group=singles[rank])
    mgr.load(e3.model, e3.optimizer, e3.scheduler, str(path))
    full = dict(e3.model.named_parameters())
    for n, p in e1.model.named_parameters():
        q = full[n]
        mom = (e1.optimizer.state[p]["exp_avg"], e3.optimizer.state[q]["exp_avg"])
        if getattr(p, "_tp_sharded", False):
            dim = 0 if p.shape[0] != q.shape[0] else 1
            k = p.shape[dim]
            q = q.narrow(dim, rank * k, k)
            mom = (mom[0], mom[1].narrow(dim, rank * k, k))
        assert torch.equal(p, q), n
        assert torch.equal(*mom), n
    assert e3.optimizer.step_count == e1.optimizer.step_count
    a = e1.train_step([{"input_ids": ids, "labels": ids}])
    b = e2.train_step([{"input_ids": ids, "labels": ids}])
    c = e3.train_step([{"input_ids": ids, "labels": ids}])
    assert torch.allclose(a["loss"], b["loss"])
    assert torch.allclose(a["loss"], c["loss"], rtol=1e-5, atol=1e-6), (a["loss"], c["loss"])
    # and back: the tp1 engine's checkpoint loads at tp2
    mgr2 = CheckpointManager(save_dir=tmp + "/tp1", save_interval=1, async_save=False)
    path2 = mgr2.save(2, *e3.state_for_save(), extra_state={"step": 2})
    e4 = TrainEngine(apply_tensor_parallel(build(cfg, seed=7), grp, sequence_parallel=True), tcfg,
                     torch.device("cpu"), dp_group=singles[rank])
    e4.tp_group = grp
    mgr2.load(e4.model, e4.optimizer, e4.scheduler, str(path2))
    full = dict(e3.model.named_parameters())
    for n, p in e4.model.named_parameters():
        q = full[n]
        if getattr(p, "_tp_sharded", False):
            dim = 0 if p.shape[0] != q.shape[0] else 1
            q = q.narrow(dim, rank * p.shape[dim], p.shape[dim])
        assert torch.equal(p, q), n
    dist.destroy_process_group()


def ep_checkpoint_worker(rank, world, port, tmp):
    """An expert-parallel checkpoint names experts by their global index, so it
    loads into the single-process layout (every rank holding all experts)."""
    init(rank, world, port)
    from nano_qwen_b200.parallel.expert_parallel import apply_expert_parallel
    from nano_qwen_b200.training.checkpoint import CheckpointManager
    from nano_qwen_b200.training.engine import TrainEngine
    cfg = tiny_cfg(moe=True)
    grp = dist.new_group(list(range(world)))
    tcfg = {"optimizer": {"lr": 1e-2}, "scheduler": {"warmup_steps": 0, "total_steps": 10}}
    # data parallel over both ranks keeps the replicated (dense) weights equal
    e1 = TrainEngine(apply_expert_parallel(build(cfg), grp, fused=False), tcfg, torch.device("cpu"))
    ids = batch(cfg, 2, 16, seed=rank)
    e1.train_step([{"input_ids": ids, "labels": ids}])
    mgr = CheckpointManager(save_dir=tmp, save_interval=1, async_save=False)
    path = mgr.save(1, *e1.state_for_save(), extra_state={"step": 1})
    # single layout, ZeRO-sharded Adam moments over the two ranks
    e2 = TrainEngine(build(cfg, seed=3), tcfg, torch.device("cpu"))
    assert e2.optimizer.sharded
    mgr.load(e2.model, e2.optimizer, e2.scheduler, str(path))
    e2.optimizer.gather_full_state()
    # the expert-parallel engine's moments are sharded too (the checkpoint
    # manager released its full views after the save)
    e1.state_for_save()
    full = dict(e2.model.named_parameters())
    e_loc = cfg.num_experts // world
    n_checked = 0
    for n, p in e1.model.named_parameters():
        if ".experts." in n:
            pre, rest = n.split(".experts.", 1)
            e, tail = rest.split(".", 1)
            n = f"{pre}.experts.{int(e) + rank * e_loc}.{tail}"
            n_checked += 1
            assert torch.equal(p, full[n]), n
            assert torch.equal(e1.optimizer.state[p]["exp_avg"], e2.optimizer.state[full[n]]["exp_avg"]), n
        else:
            assert torch.equal(p, full[n]), n
            assert torch.equal(e1.optimizer.state[p]["exp_avg"], e2.optimizer.state[full[n]]["exp_avg"]), n
    assert n_checked > 0
    e2.optimizer.release_full_state()
    e1.optimizer.release_full_state()
    dist.destroy_process_group()


# ------------------------------------------------------------------ global-batch MoE balance
def global_balance_worker(rank, world, port):
    init(rank, world, port)
    from nano_qwen_b200 import ops
    from nano_qwen_b200.training.engine import set_global_batch_balance
    cfg = tiny_cfg(moe=True)
    ids = batch(cfg, 2 * world, 16)
    m = build(cfg)
    n = set_global_batch_balance(m, None)
    assert n == cfg.num_hidden_layers
    out = m(ids[2 * rank:2 * rank + 2], labels=ids[2 * rank:2 * rank + 2])
    # oracle: f from every rank's routing counts, p from this rank's tokens
    ref = build(cfg)
    moe = ref.layers[0].feed_forward
    h = ref.embed(ids)
    resid, xn = ops.add_rms_norm(h, None, ref.layers[0].input_layernorm.weight, cfg.rms_norm_eps)
    a = ref.layers[0].attention(xn)
    resid, xn = ops.add_rms_norm(resid, a, ref.layers[0].post_attention_layernorm.weight, cfg.rms_norm_eps)
    x = xn.reshape(2 * world, 16, -1)
    w_all, idx_all, counts_all, ps_all = moe.router(x.reshape(-1, x.shape[-1]))
    mine = x[2 * rank:2 * rank + 2].reshape(-1, x.shape[-1])
    _, _, counts_loc, ps_loc = moe.router(mine)
    N = mine.shape[0]
    expect = ops.aux_loss_from_stats(counts_loc, ps_loc, N, moe.top_k, moe.num_experts,
                                     counts_all, N * world)
    # recompute layer 0's aux of the balanced model on this rank's tokens
    h2 = m.embed(ids[2 * rank:2 * rank + 2])
    r2, x2 = ops.add_rms_norm(h2, None, m.layers[0].input_layernorm.weight, cfg.rms_norm_eps)
    a2 = m.layers[0].attention(x2)
    r2, x2 = ops.add_rms_norm(r2, a2, m.layers[0].post_attention_layernorm.weight, cfg.rms_norm_eps)
    _, aux0 = m.layers[0].feed_forward(x2)
    assert torch.allclose(aux0, expect, rtol=1e-5, atol=1e-6), (float(aux0), float(expect))
    assert torch.isfinite(out["loss"])
    dist.destroy_process_group()


def rank_leave_worker(rank, world, port):
    """The last rank leaves between training steps (exits without a word); the
    survivors' step gate names it before they issue their next collective."""
    init(rank, world, port)
    from nano_qwen_b200.training.engine import TrainEngine
    from nano_qwen_b200.utils.fault import HeartbeatMonitor, PeerFailure
    store = dist.distributed_c10d._get_default_store()
    # the limit covers start-up skew between live ranks on a loaded machine
    # (a live rank that misses it would be reported as departed)
    hb = HeartbeatMonitor(store, rank, world, timeout_s=8.0, prefix="leave")
    cfg = tiny_cfg()
    eng = TrainEngine(build(cfg), {"optimizer": {"lr": 1e-3}, "scheduler": {"warmup_steps": 0}},
                      torch.device("cpu"), dp_mode="shard")
    ids = batch(cfg, 2, 16, seed=rank)
    leaver = world - 1
    dist.barrier()
    for step in range(4):
        if rank == leaver and step == 2:
            os._exit(0)  # between steps: nothing in flight, no goodbye
        try:
            hb.gate(step)
        except PeerFailure as e:
            assert rank != leaver and step == 2 and e.ranks == [leaver], (rank, step, e.ranks)
            # stop before the next collective; rank 0 hosts the store, so it
            # leaves after the other survivors have seen the failure
            store.set(f"leave/seen/{rank}", "1")
            if rank == 0:
                store.wait([f"leave/seen/{r}" for r in range(1, leaver)], datetime.timedelta(seconds=30))
            os._exit(0)
        eng.train_step([{"input_ids": ids, "labels": ids}])
    raise AssertionError("the departed rank was not detected")


def zero_checkpoint_worker(rank, world, port, tmp):
    """ZeRO shard mode keeps only this rank's slice of the Adam moments.  A
    checkpoint gathers them, and a fresh engine that loads it continues the
    run exactly: the next step's loss and every parameter match the engine
    that was never interrupted."""
    init(rank, world, port)
    from nano_qwen_b200.training.checkpoint import CheckpointManager
    from nano_qwen_b200.training.engine import TrainEngine
    cfg = tiny_cfg()
    tc = {"optimizer": {"lr": 1e-2, "grad_clip": 1.0},
          "scheduler": {"warmup_steps": 1, "total_steps": 20}}

    def engine():
        return TrainEngine(build(cfg), tc, torch.device("cpu"), dp_mode="shard")

    a = engine()
    assert a.optimizer.sharded and a.optimizer.exp_avg.numel() < a.store.numel
    data = [batch(cfg, 2, 16, seed=10 * s + rank) for s in range(4)]
    for s in range(3):
        a.train_step([{"input_ids": data[s], "labels": data[s]}])
    mgr = CheckpointManager(save_dir=tmp, async_save=False)
    m, o, sch = a.state_for_save()
    full_m = o.state[next(iter(o.state))]["exp_avg"].clone()
    d = mgr.save(3, m, o, sch)
    assert "exp_avg" not in o.state[next(iter(o.state))]  # full views released after the save
    # the saved moments are the gathered ones, nonzero outside this rank's shard
    assert full_m.abs().sum() > 0
    b = engine()
    mgr.load(b.model, b.optimizer, b.scheduler, checkpoint_dir=str(d))
    assert b.optimizer.step_count == a.optimizer.step_count
    assert torch.equal(b.optimizer.exp_avg, a.optimizer.exp_avg)
    assert torch.equal(b.optimizer.exp_avg_sq, a.optimizer.exp_avg_sq)
    ra = a.train_step([{"input_ids": data[3], "labels": data[3]}])
    rb = b.train_step([{"input_ids": data[3], "labels": data[3]}])
    assert torch.equal(ra["loss"], rb["loss"]), (ra["loss"], rb["loss"])
    a.dp.gather_master()
    b.dp.gather_master()
    assert torch.equal(a.store.master, b.store.master)
    dist.barrier()
    dist.destroy_process_group()


def pp_checkpoint_worker(rank, world, port, tmp):
    """A pipeline-parallel checkpoint names layers by their global index, so
    it loads into the single-process layout."""
    init(rank, world, port)
    from nano_qwen_b200.parallel.pipeline_parallel import apply_pipeline_parallel
    from nano_qwen_b200.training.checkpoint import CheckpointManager
    from nano_qwen_b200.training.engine import TrainEngine
    cfg = tiny_cfg(num_hidden_layers=4)
    grp = dist.new_group(list(range(world)))
    singles = [dist.new_group([r]) for r in range(world)]
    tcfg = {"optimizer": {"lr": 1e-2}, "scheduler": {"warmup_steps": 0, "total_steps": 10}}
    pm = apply_pipeline_parallel(build(cfg), grp, list(range(world)), n_microbatches=2)
    e1 = TrainEngine(pm, tcfg, torch.device("cpu"), dp_group=singles[rank])
    e1.pp_group = grp
    ids = batch(cfg, 4, 16)
    e1.train_step([{"input_ids": ids, "labels": ids}])
    mgr = CheckpointManager(save_dir=tmp, save_interval=1, async_save=False)
    path = mgr.save(1, *e1.state_for_save(), extra_state={"step": 1})
    e2 = TrainEngine(build(cfg, seed=3), tcfg, torch.device("cpu"), dp_group=singles[rank])
    mgr.load(e2.model, e2.optimizer, e2.scheduler, str(path))
    full = dict(e2.model.named_parameters())
    off = pm.stage_layers[rank][0]
    for n, p in pm.model.named_parameters():
        if n.startswith("layers."):
            i, tail = n[len("layers."):].split(".", 1)
            n = f"layers.{int(i) + off}.{tail}"
        assert torch.equal(p, full[n]), n
        assert torch.equal(e1.optimizer.state[p]["exp_avg"], e2.optimizer.state[full[n]]["exp_avg"]), n
    dist.destroy_process_group()


# ------------------------------------------------------------------ FSDP
def fsdp_worker(rank, world, port, moe, ckpt):
    """Fully sharded data parallelism (parameters, gradients and moments
    sharded; block weights gathered per use) against the ZeRO shard mode on
    the same ranks and data (itself checked against single-process
    accumulation), over three steps of two micro-batches, with and without
    activation checkpointing."""
    init(rank, world, port)
    from nano_qwen_b200.parallel.fsdp import _FREE
    from nano_qwen_b200.training.engine import TrainEngine
    cfg = tiny_cfg(moe, gradient_checkpointing=ckpt)
    tcfg = {"optimizer": {"lr": 1e-2, "grad_clip": 1.0},
            "scheduler": {"warmup_steps": 0, "total_steps": 10}}
    ref = TrainEngine(build(cfg), tcfg, torch.device("cpu"), dp_mode="shard")
    fs = TrainEngine(build(cfg), dict(tcfg, distributed={"shard_params": True}), torch.device("cpu"))
    st = fs.store
    assert st.mode == "fsdp" and fs.dp is st
    total = sum(p.numel() for p in fs.model.parameters())
    # every per-rank buffer holds about 1/world of the parameters
    assert st.master.numel() == fs.optimizer.exp_avg.numel() == st.grad.numel()
    assert st.master.numel() <= total / world + 64 * len(st.units), (st.master.numel(), total)
    for step in range(3):
        ids = batch(cfg, 2 * world, 16, seed=100 + step)
        mine = [{"input_ids": ids[2 * rank + i:2 * rank + i + 1],
                 "labels": ids[2 * rank + i:2 * rank + i + 1]} for i in range(2)]
        r = ref.train_step(mine)
        f = fs.train_step(mine)
        close(f["loss"], r["loss"], 1e-5, "loss")
        close(f["grad_norm"], r["grad_norm"], 1e-4, "grad norm")
        if moe:
            close(f["aux_loss"], r["aux_loss"], 1e-5, "aux loss")
        # block weights are released between steps
        assert all(u.state == _FREE for u in st.block_units[:-1])
        assert not any(u.grad_live for u in st.units)
    ref.state_for_save()
    fs.state_for_save()
    for (n, p), (_, q) in zip(fs.model.named_parameters(), ref.model.named_parameters()):
        assert p.dtype == torch.float32 and p.shape == q.shape, n
        close(p, q, 1e-5, n)
    fs.optimizer.release_full_state()
    dist.destroy_process_group()


def fsdp_ep_worker(rank, world, port, ep):
    """Fully sharded parameters with expert parallelism: dense matrices
    sharded over the data-parallel group, each block's local experts over
    the ranks that hold the same experts; against the replicated EP engine
    (itself checked against the single-process model) on the same layout."""
    init(rank, world, port)
    from nano_qwen_b200.parallel.manager import ParallelConfig, ParallelismManager
    from nano_qwen_b200.training.engine import TrainEngine
    cfg = tiny_cfg(moe=True)
    tcfg = {"optimizer": {"lr": 1e-2, "grad_clip": 1.0},
            "scheduler": {"warmup_steps": 0, "total_steps": 10}}

    def engine(shard):
        pm = ParallelismManager(ParallelConfig(ep_size=ep, ep_fused=False))
        m = pm.apply_parallelism(build(cfg))
        return TrainEngine(m, dict(tcfg, distributed={"shard_params": shard}), torch.device("cpu"),
                           parallel=pm)

    ref, fs = engine(False), engine(True)
    assert fs.store.mode == "fsdp"
    xu = [u for u in fs.store.units if u.name.endswith(".experts")]
    assert xu and all(u.world == world // ep for u in xu), [(u.name, u.world) for u in xu]
    for step in range(3):
        ids = batch(cfg, 2 * world, 16, seed=300 + step)
        mine = [{"input_ids": ids[2 * rank:2 * rank + 2], "labels": ids[2 * rank:2 * rank + 2]}]
        r = ref.train_step(mine)
        f = fs.train_step(mine)
        close(f["loss"], r["loss"], 1e-5, "loss")
        close(f["grad_norm"], r["grad_norm"], 1e-4, "grad norm")
    ref.state_for_save()
    fs.state_for_save()
    for (n, p), (_, q) in zip(fs.model.named_parameters(), ref.model.named_parameters()):
        close(p, q, 1e-5, n)
    fs.optimizer.release_full_state()
    dist.destroy_process_group()


def fsdp_api_worker(rank, world, port):
    """The reference's calls (``apply_fsdp2`` per block + root, then a plain
    loop: forward, backward, clip, step) on the fully sharded store give the
    ZeRO engine's losses and weights."""
    init(rank, world, port)
    from nano_qwen_b200.parallel.fsdp import FSDPAdamW, apply_fsdp2, get_mixed_precision_policy
    from nano_qwen_b200.training.engine import TrainEngine
    from nano_qwen_b200.training.optimizer import build_optimizer
    cfg = tiny_cfg()
    tcfg = {"optimizer": {"lr": 1e-2, "grad_clip": 1.0, "weight_decay": 0.1},
            "scheduler": {"warmup_steps": 0, "total_steps": 10}}
    ref = TrainEngine(build(cfg), tcfg, torch.device("cpu"), dp_mode="shard")
    model = apply_fsdp2(build(cfg), None, get_mixed_precision_policy("bfloat16"))
    opt = build_optimizer(model, lr=1e-2, weight_decay=0.1)
    assert isinstance(opt, FSDPAdamW)
    for step in range(3):
        ids = batch(cfg, 2 * world, 16, seed=200 + step)
        mine = ids[2 * rank:2 * rank + 2]
        lrs = [g["lr"] for g in ref.optimizer.param_groups]   # what the engine's step uses
        r = ref.train_step([{"input_ids": mine, "labels": mine}])
        loss = model(mine, labels=mine)["loss"]
        loss.backward()
        norm = opt.clip_grad_norm_(1.0)
        for g, lr in zip(opt.param_groups, lrs):
            g["lr"] = lr
        opt.step()
        opt.zero_grad()
        close(loss.detach(), r["loss"], 1e-5, "loss")
        close(norm, r["grad_norm"], 1e-4, "grad norm")
    dist.destroy_process_group()


def fsdp_checkpoint_worker(rank, world, port, tmp):
    """A fully sharded run saves the single-process state (DCP): a fresh
    fully sharded engine resumes it exactly, and a 1-rank engine loads the
    same weights and moments."""
    init(rank, world, port)
    from nano_qwen_b200.training.checkpoint import CheckpointManager
    from nano_qwen_b200.training.engine import TrainEngine
    cfg = tiny_cfg()
    tc = {"optimizer": {"lr": 1e-2, "grad_clip": 1.0},
          "scheduler": {"warmup_steps": 1, "total_steps": 20},
          "distributed": {"shard_params": True}}

    def engine(**kw):
        return TrainEngine(build(cfg, seed=kw.pop("seed", 0)), tc, torch.device("cpu"), **kw)

    a = engine()
    data = [batch(cfg, 2, 16, seed=10 * s + rank) for s in range(4)]
    for s in range(3):
        a.train_step([{"input_ids": data[s], "labels": data[s]}])
    mgr = CheckpointManager(save_dir=tmp, async_save=True)
    d = mgr.save(3, *a.state_for_save())
    # the save completed in the call (the parameters were bound to the gathered
    # tensors) and the parameters are views of the gathered units again
    assert a.optimizer._full is None and mgr._pending is None
    for p in a.model.parameters():
        assert p.data_ptr() == a.store._pviews[id(p)].data_ptr()
    p0 = next(iter(a.model.parameters()))
    assert p0.dtype == torch.float32 and "exp_avg" not in a.optimizer.state[p0]  # released
    b = engine(seed=3)
    mgr.load(b.model, b.optimizer, b.scheduler, checkpoint_dir=str(d))
    assert b.optimizer.step_count == a.optimizer.step_count
    assert torch.equal(b.store.master, a.store.master)
    assert torch.equal(b.optimizer.exp_avg, a.optimizer.exp_avg)
    assert torch.equal(b.optimizer.exp_avg_sq, a.optimizer.exp_avg_sq)
    ra = a.train_step([{"input_ids": data[3], "labels": data[3]}])
    rb = b.train_step([{"input_ids": data[3], "labels": data[3]}])
    assert torch.equal(ra["loss"], rb["loss"]), (ra["loss"], rb["loss"])
    # the 1-rank (unsharded) layout reads the same checkpoint
    singles = [dist.new_group([r]) for r in range(world)]
    c = TrainEngine(build(cfg, seed=9), dict(tc, distributed={}), torch.device("cpu"),
                    dp_group=singles[rank])
    mgr.load(c.model, c.optimizer, c.scheduler, checkpoint_dir=str(d))
    a2 = engine(seed=4)
    mgr.load(a2.model, a2.optimizer, a2.scheduler, checkpoint_dir=str(d))
    a2.state_for_save()
    full = dict(c.model.named_parameters())
    for n, p in a2.model.named_parameters():
        assert torch.equal(p, full[n]), n
        assert torch.equal(a2.optimizer.state[p]["exp_avg"], c.optimizer.state[full[n]]["exp_avg"]), n
    a2.optimizer.release_full_state()
    dist.barrier()
    dist.destroy_process_group()


def sft_parallel_worker(rank, world, port, tmp, axis):
    """The SFT phase through the CLI with a model-parallel layout from the
    training YAML (as pretraining takes it): two steps and a checkpoint."""
    import yaml
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    torch.set_num_threads(1)
    os.chdir(tmp)
    from nano_qwen_b200.cli import main
    model = dict(hidden_size=64, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                 head_dim=16, intermediate_size=128, vocab_size=300, max_position_embeddings=256,
                 tie_word_embeddings=True)
    train = {"optimizer": {"lr": 1e-3}, "scheduler": {"warmup_steps": 1, "total_steps": 4},
             "batch": {"micro_batch_size": 2, "gradient_accumulation_steps": 1, "max_seq_len": 64},
             "checkpoint": {"save_interval": 2, "save_dir": "ck", "async_save": False},
             "logging": {"log_interval": 1, "tensorboard_enabled": False},
             "distributed": {axis: world}}
    if rank == 0:
        with open("m.yaml", "w") as f:
            yaml.safe_dump(model, f)
        with open("t.yaml", "w") as f:
            yaml.safe_dump(train, f)
    else:
        import time
        while not os.path.exists("t.yaml"):
            time.sleep(0.05)
        time.sleep(0.2)
    assert main(["sft", "--model-config", "m.yaml", "--training-config", "t.yaml",
                 "--max-steps", "2", "--max-samples", "8"]) == 0
    assert os.path.isdir("ck/step_00000002")
    if dist.is_initialized():
        dist.destroy_process_group()


# ----------------------------------------------- peer-memory ZeRO host code
def _install_fake_peer(tmp):
    """Route ``parallel.peer_dp`` to the file-backed stand-in (``fake_peer``)."""
    import fake_peer
    from nano_qwen_b200.parallel import peer_dp
    peer_dp.symmetric_available = lambda group=None: True
    peer_dp.SymmetricAllocator = fake_peer.make_allocator_factory(tmp)
    peer_dp.ext = lambda: fake_peer.FakeZeroExt()
    torch.cuda.synchronize = lambda *a, **k: None
    # the peer engines (their stores come from the symmetric allocator) get
    # a bf16 compute copy, as on the GPU
    from nano_qwen_b200.training import engine as engine_mod
    from nano_qwen_b200.training.optimizer import attach_param_store
    engine_mod.attach_param_store = lambda m, **kw: attach_param_store(
        m, torch.bfloat16 if kw.get("alloc") is not None else None, **kw)
    # the CPU forward reads the fp32 master, which the step updates only in
    # this rank's ranges (the GPU forward reads the all-gathered bf16 copy):
    # complete it after each step
    if not getattr(peer_dp.PeerDataParallel, "_fake_gathers", False):
        step = peer_dp.PeerDataParallel.fused_step

        def fused_step(self, *a, **k):
            norm = step(self, *a, **k)
            self.gather_master()
            return norm
        peer_dp.PeerDataParallel.fused_step = fused_step
        peer_dp.PeerDataParallel._fake_gathers = True


def peer_dp_fake_worker(rank, world, port, tmp):
    """The host code of the fused data-parallel step (``PeerDataParallel``:
    epochs, shard bounds, the sharded moments, ``fused_step``, checkpointing)
    on Gloo CPU ranks over a file-backed stand-in for symmetric memory and
    restated kernels (``fake_peer``).  Against the NCCL-style ZeRO shard
    engine on the same data: losses, norms and weights for three steps, then
    a checkpoint that a fresh peer engine resumes exactly."""
    init(rank, world, port)
    import fake_peer
    from nano_qwen_b200.parallel import peer_dp
    from nano_qwen_b200.training import engine as engine_mod
    from nano_qwen_b200.training.checkpoint import CheckpointManager
    from nano_qwen_b200.training.engine import TrainEngine
    from nano_qwen_b200.training.optimizer import attach_param_store

    _install_fake_peer(tmp)
    cfg = tiny_cfg()
    tc = {"optimizer": {"lr": 1e-2, "grad_clip": 1.0},
          "scheduler": {"warmup_steps": 1, "total_steps": 20}}
    ref = TrainEngine(build(cfg), tc, torch.device("cpu"), dp_mode="shard")
    a = TrainEngine(build(cfg), tc, torch.device("cpu"), dp_mode="p2p")
    assert isinstance(a.dp, peer_dp.PeerDataParallel) and a.optimizer.sharded
    data = [batch(cfg, 2, 16, seed=10 * s + rank) for s in range(5)]
    for s in range(3):
        r = ref.train_step([{"input_ids": data[s], "labels": data[s]}])
        o = a.train_step([{"input_ids": data[s], "labels": data[s]}])
        close(o["loss"], r["loss"], 1e-5, "loss")
        close(o["grad_norm"], r["grad_norm"], 1e-5, "grad norm")
        # the CPU forward reads the fp32 master, which the step updates only in
        # this rank's shard (the GPU forward reads the all-gathered bf16 copy)
        a.dp.gather_master()
        close(a.store.master, ref.store.master, 1e-5, "master")
        comp = a.store.compute.float()
        assert torch.equal(comp, a.store.master.to(torch.bfloat16).float()), "compute copy"
    mgr = CheckpointManager(save_dir=os.path.join(tmp, "ck"), async_save=False)
    d = mgr.save(3, *a.state_for_save())
    b = TrainEngine(build(cfg, seed=4), tc, torch.device("cpu"), dp_mode="p2p")
    mgr.load(b.model, b.optimizer, b.scheduler, checkpoint_dir=str(d))
    assert torch.equal(b.optimizer.exp_avg, a.optimizer.exp_avg)
    assert torch.equal(b.optimizer.exp_avg_sq, a.optimizer.exp_avg_sq)
    ra = a.train_step([{"input_ids": data[3], "labels": data[3]}])
    rb = b.train_step([{"input_ids": data[3], "labels": data[3]}])
    assert torch.equal(ra["loss"], rb["loss"]), (ra["loss"], rb["loss"])
    dist.barrier()
    dist.destroy_process_group()


def fsdp_tp_worker(rank, world, port, tp, moe):
    """Fully sharded parameters with tensor (+ sequence) parallelism: the
    tensor shards sharded again over the data-parallel ranks, partial
    replicated gradients summed over the tensor group before each unit's
    reduce-scatter, duplicates left out of the gradient norm; against the
    ZeRO engine on the same tp x dp layout."""
    init(rank, world, port)
    from nano_qwen_b200.parallel.manager import ParallelConfig, ParallelismManager
    from nano_qwen_b200.training.engine import TrainEngine
    cfg = tiny_cfg(moe)
    tcfg = {"optimizer": {"lr": 1e-2, "grad_clip": 1.0},
            "scheduler": {"warmup_steps": 0, "total_steps": 10}}

    def engine(shard):
        pm = ParallelismManager(ParallelConfig(tp_size=tp, tp_fused=False))
        m = pm.apply_parallelism(build(cfg))
        return TrainEngine(m, dict(tcfg, distributed={"shard_params": shard}), torch.device("cpu"),
                           parallel=pm), pm

    (ref, pm), (fs, _) = engine(False), engine(True)
    assert fs.store.mode == "fsdp" and fs.store.tp_group is not None
    d = pm.coords["dp"]
    for step in range(3):
        ids = batch(cfg, 2 * (world // tp), 16, seed=400 + step)
        mine = [{"input_ids": ids[2 * d:2 * d + 2], "labels": ids[2 * d:2 * d + 2]}]
        r = ref.train_step(mine)
        f = fs.train_step(mine)
        close(f["loss"], r["loss"], 1e-5, "loss")
        close(f["grad_norm"], r["grad_norm"], 1e-4, "grad norm")
    ref.state_for_save()
    fs.state_for_save()
    for (n, p), (_, q) in zip(fs.model.named_parameters(), ref.model.named_parameters()):
        close(p, q, 1e-5, n)
    fs.optimizer.release_full_state()
    dist.destroy_process_group()


def tp_engine_worker(rank, world, port):
    """A training engine under tensor parallelism over every rank (one data-
    parallel replica): no data-parallel reduction runs (the manager has no
    group for a size-1 axis, which must not mean the default group), and
    three steps match the single-process engine on the same batch."""
    init(rank, world, port)
    from nano_qwen_b200.parallel.manager import ParallelConfig, ParallelismManager
    from nano_qwen_b200.training.engine import TrainEngine
    cfg = tiny_cfg()
    tcfg = {"optimizer": {"lr": 1e-2, "grad_clip": 1.0},
            "scheduler": {"warmup_steps": 0, "total_steps": 10}}
    singles = [dist.new_group([r]) for r in range(world)]
    ref = TrainEngine(build(cfg), tcfg, torch.device("cpu"), dp_group=singles[rank])
    pm = ParallelismManager(ParallelConfig(tp_size=world, tp_fused=False))
    eng = TrainEngine(pm.apply_parallelism(build(cfg)), tcfg, torch.device("cpu"), parallel=pm)
    assert eng.dp is None
    for step in range(3):
        ids = batch(cfg, 2, 16, seed=500 + step)
        r = ref.train_step([{"input_ids": ids, "labels": ids}])
        o = eng.train_step([{"input_ids": ids, "labels": ids}])
        close(o["loss"], r["loss"], 1e-5, "loss")
        close(o["grad_norm"], r["grad_norm"], 1e-4, "grad norm")
    dist.destroy_process_group()


def layouts_worker(rank, world, port, layouts):
    """Every (name, layout) in ``layouts`` in one spawned job (the process
    group is set up once); a failure names its layout."""
    init(rank, world, port)
    for name, layout in layouts:
        try:
            _layout_case(rank, world, layout)
        except AssertionError as e:
            raise AssertionError(f"layout {name}: {e}") from e
    dist.destroy_process_group()


def layout_worker(rank, world, port, layout):
    init(rank, world, port)
    _layout_case(rank, world, layout)
    dist.destroy_process_group()


def _layout_case(rank, world, layout):
    """The training engine on one parallel layout built by the
    ``ParallelismManager`` (``layout``: ParallelConfig fields plus ``moe``
    and ``shard_params``), two steps against the single-process engine on
    the same global batch (the data-parallel ranks' slices as its
    micro-batches): losses and gradient norms agree."""
    from nano_qwen_b200.parallel.manager import ParallelConfig, ParallelismManager
    from nano_qwen_b200.training.engine import TrainEngine
    layout = dict(layout)
    moe = layout.pop("moe", False)
    shard = layout.pop("shard_params", False)
    accum = layout.pop("accum", 1)
    tied = layout.pop("tied", False)
    # routing statistics are per rank under most layouts: compare without the
    # aux term, except for the global-batch balance, whose statistics are the
    # full batch's (then the reference runs the full batch as one micro-batch)
    balance = layout.pop("balance", False)
    docs = layout.pop("docs", False)
    pad = layout.pop("pad", False)
    dp_mode = layout.pop("dp_mode", None)
    cfg_mode = layout.pop("dp_mode_cfg", None)   # named in the training config instead
    expect_nccl = layout.pop("expect_nccl", False)
    overlap = layout.pop("overlap", False)
    cfg = tiny_cfg(moe, router_aux_loss_coef=0.05 if balance else 0.0, num_hidden_layers=2,
                   tie_word_embeddings=tied)
    tcfg = {"optimizer": {"lr": 1e-2, "grad_clip": 1.0},
            "scheduler": {"warmup_steps": 0, "total_steps": 10},
            "moe": {"global_batch_balance": balance}}
    singles = [dist.new_group([r]) for r in range(world)]
    ref = TrainEngine(build(cfg), tcfg, torch.device("cpu"), dp_group=singles[rank])
    pm = ParallelismManager(ParallelConfig(tp_fused=False, ep_fused=False, **layout))
    dcfg = {"shard_params": shard, "overlap_grad_reduce": overlap}
    if cfg_mode:
        dcfg["dp_mode"] = cfg_mode
    eng = TrainEngine(pm.apply_parallelism(build(cfg)), dict(tcfg, distributed=dcfg),
                      torch.device("cpu"), dp_mode=dp_mode, parallel=pm)
    _check_peer_step(eng, dp_mode or cfg_mode)
    if expect_nccl:   # the configured default (dp_comm: p2p) under model parallelism
        from nano_qwen_b200.parallel.peer_dp import PeerDataParallel
        assert eng.dp is not None and not isinstance(eng.dp, PeerDataParallel), type(eng.dp)
    dp = pm.config.dp_size
    d = pm.coords["dp"]
    B = 4
    for step in range(2):   # the second step checks the first update
        ids = batch(cfg, B * dp, 16, seed=600 + step)
        c = B // accum
        full = [{"input_ids": ids[c * i:c * (i + 1)], "labels": ids[c * i:c * (i + 1)]}
                for i in range(dp * accum)]
        if docs:   # packed documents: each token attends within its own document
            gd = torch.Generator().manual_seed(900 + step)
            cuts = (torch.rand(ids.shape, generator=gd) < 0.2).long()
            cuts[:, 0] = 0
            dids = cuts.cumsum(1)
            for i, mb in enumerate(full):
                mb["doc_ids"] = dids[c * i:c * (i + 1)]
        if pad:    # right padding of uneven length: masked keys, ignored targets
            gp = torch.Generator().manual_seed(950 + step)
            lens = torch.randint(6, 17, (ids.shape[0],), generator=gp)
            am = (torch.arange(ids.shape[1])[None, :] < lens[:, None]).long()
            lab = torch.where(am.bool(), ids, torch.full_like(ids, -100))
            for i, mb in enumerate(full):
                mb["attention_mask"] = am[c * i:c * (i + 1)]
                mb["labels"] = lab[c * i:c * (i + 1)]
        if balance:
            r = ref.train_step([{"input_ids": ids, "labels": ids}])
        else:
            r = ref.train_step(full)
        o = eng.train_step(full[d * accum:(d + 1) * accum])
        if overlap:   # every block's span was reduced during the backward
            assert eng.dp.last_overlapped == len(eng.dp._hooked) > 0, \
                (eng.dp.last_overlapped, len(eng.dp._hooked))
        # the engine reports its replica's loss; the mean over the replicas
        # (every rank of a replica reports the same value) is the global one
        loss = o["loss"].detach().clone()
        dist.all_reduce(loss)
        close(loss / world, r["loss"], 1e-5, f"loss step {step}")
        close(o["grad_norm"], r["grad_norm"], 1e-4, f"grad norm step {step}")


def _check_peer_step(eng, dp_mode):
    """A layout that asks for the peer-memory step gets it; a data-parallel
    step that keeps its state in pieces owns a partition of the store."""
    if dp_mode == "p2p":
        from nano_qwen_b200.parallel.peer_dp import PeerDataParallel
        assert isinstance(eng.dp, PeerDataParallel), type(eng.dp)
        assert eng.optimizer.sharded
    if getattr(eng.dp, "piecewise", False):
        # the owned ranges partition the store: every dense element once over
        # the data-parallel group, every expert element once per expert set;
        # the Adam moments hold exactly the owned elements
        dp, st = eng.dp, eng.store
        own = dp.owned_ranges()
        n_own = sum(hi - lo for lo, hi in own)
        assert eng.optimizer.exp_avg.numel() == n_own
        xb, xe = dp.expert_span or (0, 0)
        x_world = (dp.split[2][3] if getattr(dp, "split", None) is not None
                   else getattr(dp, "x_world", 1))
        for lo, hi in own:
            assert hi <= xb or lo >= xe or (xb <= lo and hi <= xe), (lo, hi, dp.expert_span)
        tot = torch.tensor([n_own], dtype=torch.float64)
        dist.all_reduce(tot, group=dp.group)
        sets = dp.world // x_world if dp.expert_span is not None else 1
        assert int(tot) == st.numel - (xe - xb) + (xe - xb) * sets, (int(tot), st.numel, xe - xb)


def peer_layouts_worker(rank, world, port, cases, tmp):
    """``layouts_worker`` with the peer-memory step's host code running over
    the file-backed stand-in for symmetric memory (``fake_peer``)."""
    init(rank, world, port)
    _install_fake_peer(tmp)
    for name, layout in cases:
        try:
            _layout_case(rank, world, layout)
        except AssertionError as e:
            raise AssertionError(f"layout {name}: {e}") from e
    dist.destroy_process_group()


def layout_ckpts_worker(rank, world, port, cases, tmp):
    """Every (name, layout, from_single) checkpoint case of one world size
    in one spawned job; a failure names its case."""
    init(rank, world, port)
    if any(lay.get("dp_mode") == "p2p" for _, lay, _ in cases):
        _install_fake_peer(os.path.join(tmp, "peer"))
    for k, (name, layout, from_single) in enumerate(cases):
        try:
            _layout_ckpt_case(rank, world, layout, os.path.join(tmp, f"case{k}"), from_single)
        except AssertionError as e:
            raise AssertionError(f"layout {name} (from_single={from_single}): {e}") from e
    dist.destroy_process_group()


def _layout_ckpt_case(rank, world, layout, tmp, from_single=False):
    """A checkpoint written by an engine on any manager layout loads into the
    single-process engine, which then continues exactly like the layout
    engine: two more steps with equal losses and gradient norms (weights,
    Adam moments and step counts all carried over)."""
    from nano_qwen_b200.parallel.manager import ParallelConfig, ParallelismManager
    from nano_qwen_b200.training.checkpoint import CheckpointManager
    from nano_qwen_b200.training.engine import TrainEngine
    layout = dict(layout)
    moe = layout.pop("moe", False)
    shard = layout.pop("shard_params", False)
    dp_mode = layout.pop("dp_mode", None)
    overlap = layout.pop("overlap", False)
    cfg = tiny_cfg(moe, router_aux_loss_coef=0.0, num_hidden_layers=4)
    tcfg = {"optimizer": {"lr": 1e-2, "grad_clip": 1.0},
            "scheduler": {"warmup_steps": 0, "total_steps": 10}, "moe": {"global_batch_balance": False}}
    singles = [dist.new_group([r]) for r in range(world)]
    pm = ParallelismManager(ParallelConfig(tp_fused=False, ep_fused=False, **layout))
    eng = TrainEngine(pm.apply_parallelism(build(cfg)),
                      dict(tcfg, distributed={"shard_params": shard, "overlap_grad_reduce": overlap}), torch.device("cpu"),
                      dp_mode=dp_mode, parallel=pm)
    _check_peer_step(eng, dp_mode)
    dp, d, B = pm.config.dp_size, pm.coords["dp"], 4

    def data(step):
        ids = batch(cfg, B * dp, 16, seed=700 + step)
        return [{"input_ids": ids[B * i:B * (i + 1)], "labels": ids[B * i:B * (i + 1)]} for i in range(dp)]

    one = TrainEngine(build(cfg, seed=11), tcfg, torch.device("cpu"), dp_group=singles[rank])
    mgr = CheckpointManager(save_dir=os.path.join(tmp, "ck"), async_save=False)
    if from_single:   # the other direction: one process writes, the layout reads
        for step in range(2):
            one.train_step(data(step))
        # every rank holds the same single-process state; DCP writes it once
        path = mgr.save(2, *one.state_for_save(), extra_state={"step": 2})
        mgr.load(eng.model, eng.optimizer, eng.scheduler, str(path))
        assert eng.optimizer.step_count == 2
    else:
        for step in range(2):
            eng.train_step([data(step)[d]])
        path = mgr.save(2, *eng.state_for_save(), extra_state={"step": 2})
        mgr.load(one.model, one.optimizer, one.scheduler, str(path))
        assert one.optimizer.step_count == 2
    for step in (2, 3):
        full = data(step)
        r = one.train_step(full)
        o = eng.train_step([full[d]])
        loss = o["loss"].detach().clone()
        dist.all_reduce(loss)
        close(loss / world, r["loss"], 1e-5, f"loss step {step}")
        close(o["grad_norm"], r["grad_norm"], 1e-4, f"grad norm step {step}")
    dist.barrier()


def dpo_layout_worker(rank, world, port, shard):
    """DPO over two data-parallel ranks (ZeRO or fully sharded) against one
    process on all pairs: per-step gradient norms and the replica-mean
    loss."""
    init(rank, world, port)
    from nano_qwen_b200.training.dpo import DPOTrainer
    cfg = tiny_cfg()
    tc = {"dpo": {"beta": 0.3}, "optimizer": {"lr": 1e-2, "grad_clip": 1.0},
          "scheduler": {"warmup_steps": 0, "total_steps": 10}}
    singles = [dist.new_group([r]) for r in range(world)]
    one = DPOTrainer(build(cfg), build(cfg, seed=5), tc, torch.device("cpu"), dp_group=singles[rank])
    two = DPOTrainer(build(cfg), build(cfg, seed=5), dict(tc, distributed={"shard_params": shard}),
                     torch.device("cpu"))
    for step in range(3):
        g = torch.Generator().manual_seed(800 + step)
        c = torch.randint(0, cfg.vocab_size, (2 * world, 12), generator=g)
        r = torch.randint(0, cfg.vocab_size, (2 * world, 12), generator=g)
        a = one.train_step(c, r, c.clone(), r.clone())
        sl = slice(2 * rank, 2 * rank + 2)
        b = two.train_step(c[sl], r[sl], c[sl].clone(), r[sl].clone())
        loss = torch.tensor(b["loss"])
        dist.all_reduce(loss)
        assert abs(float(loss) / world - a["loss"]) < 1e-5 * max(1.0, abs(a["loss"])), (loss, a)
        assert abs(b["grad_norm"] - a["grad_norm"]) < 1e-4 * a["grad_norm"], (b, a)
    dist.destroy_process_group()
