"""Pretraining entry point (stages 1-3).

Same entry point and training-YAML surface as the reference
(``run_pretraining(model_config_path, training_config_path, resume_from)``;
reference: training/pretrain.py:222-266).  Differences: the ``--stage`` flag is
honoured (stage 3 enables YARN long-context scaling when the model config has
no ``rope_scaling``), the step loop is the ``TrainEngine`` (no per-micro-step
host syncs), throughput is global tokens per device-timed second and MFU is
reported against the measured B200 peak.
"""

from __future__ import annotations

import time
from typing import Optional

import torch
import yaml
from torch.utils.data import DataLoader

from ..config import ModelConfig
from ..data.collator import TextCollator
from ..data.dataset import PackedTextDataset
from ..data.sampler import DistributedSampler
from ..models.transformer import Qwen3Model
from ..parallel.comm import (get_local_rank, init_distributed, is_main_process,
                             max_over_ranks)
from ..utils.flops import mfu
from .checkpoint import CheckpointManager, resolve_resume
from .engine import TrainEngine
from .logger import TrainingLogger


def load_training_config(path: Optional[str]) -> dict:
    if path is None:
        return {}
    with open(path) as f:
        return yaml.safe_load(f) or {}


def pick_device() -> torch.device:
    if torch.cuda.is_available():
        return torch.device("cuda", get_local_rank())
    return torch.device("cpu")


def compute_mfu(model_params: int, tokens_per_sec: float, num_gpus: int,
                gpu_flops: Optional[float] = None) -> float:
    """6*N FLOPs/token MFU (reference helper, training/pretrain.py:47-57), with
    the peak defaulting to the measured B200 bf16 figure."""
    from ..utils.flops import peak_flops
    peak = (gpu_flops or peak_flops()) * num_gpus
    return 6 * model_params * tokens_per_sec / peak if peak > 0 else 0.0


def build_parallel(training_config: dict, world_size: int):
    """A ``ParallelismManager`` when the ``distributed`` section asks for any
    model-parallel axis (tp/pp/ep/cp > 1); plain data parallelism otherwise."""
    d = training_config.get("distributed", {}) or {}
    sizes = {k: int(d.get(k, 1) or 1) for k in ("tp_size", "pp_size", "ep_size", "cp_size")}
    if world_size <= 1 or all(v == 1 for v in sizes.values()):
        return None
    from ..parallel.manager import ParallelConfig, ParallelismManager
    pc = ParallelConfig(dp_size=int(d.get("dp_size", -1) or -1), **sizes,
                        fsdp_enabled=bool(d.get("fsdp_enabled", True)),
                        sequence_parallel=bool(d.get("sequence_parallel", True)),
                        pp_microbatches=int(d.get("pp_microbatches", 4)),
                        cp_mode=str(d.get("cp_mode", "allgather")))
    return ParallelismManager(pc)


class PreTrainer:
    def __init__(self, model_config: ModelConfig, training_config: dict, stage: int = 1):
        self.model_config = model_config
        self.cfg = training_config
        self.rank, self.world_size = init_distributed()
        self.device = pick_device()
        if stage == 3 and model_config.rope_scaling is None:
            model_config.rope_scaling = {"type": "yarn", "factor": 4.0,
                                         "original_max_position_embeddings":
                                             model_config.max_position_embeddings}
            model_config.max_position_embeddings *= 4
        torch.manual_seed(self.cfg.get("seed", 0))
        model = Qwen3Model(model_config)
        if is_main_process():
            c = model.count_parameters()
            print(f"Model parameters: {c['total']:,} total, {c['trainable']:,} trainable")
        self.parallel = build_parallel(training_config, self.world_size)
        self.dp_rank, self.dp_size = self.rank, self.world_size
        if self.parallel is not None:
            model = self.parallel.apply_parallelism(model.to(self.device))
            self.dp_rank = self.parallel.coords["dp"]
            self.dp_size = self.parallel.config.dp_size
        self.engine = TrainEngine(model, training_config, self.device, parallel=self.parallel)
        self.model = self.engine.model
        self.optimizer = self.engine.optimizer
        self.scheduler = self.engine.scheduler
        ck = training_config.get("checkpoint", {}) or {}
        self.ckpt_mgr = CheckpointManager(save_dir=ck.get("save_dir", "checkpoints"),
                                          save_interval=ck.get("save_interval", 1000),
                                          async_save=ck.get("async_save", True))
        lg = training_config.get("logging", {}) or {}
        self.logger = TrainingLogger(wandb_project=lg.get("wandb_project"),
                                     wandb_enabled=lg.get("wandb_enabled", False),
                                     tensorboard_dir=lg.get("tensorboard_dir"),
                                     tensorboard_enabled=lg.get("tensorboard_enabled", True),
                                     log_interval=lg.get("log_interval", 10))
        self.grad_accum_steps = (training_config.get("batch", {}) or {}).get(
            "gradient_accumulation_steps", 1)
        # optional torch.profiler window over training steps (training YAML
        # ``profiling``: enabled / wait / warmup / active / dir)
        from ..utils.tracing import step_profiler_from_config
        self.step_profiler = step_profiler_from_config(training_config.get("profiling"),
                                                       rank=self.rank)
        # optional failure detection between steps (training YAML ``fault``:
        # ``step_gate_timeout_s``): every rank announces each step in the c10d
        # store and a rank that left is named before the next collective
        self.step_gate = None
        gate_s = (training_config.get("fault", {}) or {}).get("step_gate_timeout_s")
        if gate_s and self.world_size > 1:
            import torch.distributed as dist
            from ..utils.fault import HeartbeatMonitor
            self.step_gate = HeartbeatMonitor(dist.distributed_c10d._get_default_store(), self.rank,
                                              self.world_size, timeout_s=float(gate_s), prefix="nq_gate")

    def train(self, dataloader, total_steps: int, start_step: int = 0, sampler=None):
        step = start_step
        it = iter(dataloader)
        cuda = self.device.type == "cuda"
        seq_len = None
        tokens_window = 0
        t_window = 0.0
        while step < total_steps:
            mbs = []
            for _ in range(self.grad_accum_steps):
                try:
                    b = next(it)
                except StopIteration:
                    it = iter(dataloader)
                    b = next(it)
                mbs.append({k: v.to(self.device, non_blocking=True) for k, v in b.items()})
            seq_len = mbs[0]["input_ids"].shape[1]
            ntok = sum(m["input_ids"].numel() for m in mbs) * self.dp_size
            if cuda:
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
            if self.step_gate is not None:
                self.step_gate.gate(step)
            t0 = time.perf_counter()
            if self.step_profiler is not None:
                with self.step_profiler.step(step):
                    out = self.engine.train_step(mbs)
            else:
                out = self.engine.train_step(mbs)
            step += 1
            if cuda:
                e1.record()
            do_log = step % self.logger.log_interval == 0
            if do_log:
                if cuda:
                    e1.synchronize()
                    dt = e0.elapsed_time(e1) / 1e3
                else:
                    dt = time.perf_counter() - t0
                dt = max_over_ranks(dt)
                tps = ntok / dt
                n_params = sum(p.numel() for p in self.model.parameters())
                # device scalars: the logger reads them back in one copy
                self.logger.log_step(step=step, loss=out["loss"],
                                     lr=self.scheduler.get_last_lr()[0],
                                     grad_norm=out["grad_norm"], tokens_per_sec=tps,
                                     aux_loss=out["aux_loss"],
                                     mfu=mfu(self.model_config, seq_len, tps, self.world_size))
            if self.ckpt_mgr.should_save(step):
                model, opt, sch = self.engine.state_for_save()
                if sampler is not None:
                    sampler.set_start_index(step * self.grad_accum_steps * dataloader.batch_size)
                self.ckpt_mgr.save(step, model, opt, sch, extra_state={"step": step},
                                   sampler=sampler)
        self.ckpt_mgr.wait()
        if is_main_process():
            print("Training complete.")
        self.logger.finish()


def run_pretraining(model_config_path: str, training_config_path: str,
                    resume_from: Optional[str] = None, stage: int = 1,
                    max_steps: Optional[int] = None):
    model_config = ModelConfig.from_yaml(model_config_path)
    tcfg = load_training_config(training_config_path)
    trainer = PreTrainer(model_config, tcfg, stage=stage)
    data_cfg = tcfg.get("data", {}) or {}
    batch_cfg = tcfg.get("batch", {}) or {}
    dataset = PackedTextDataset(data_dir=data_cfg.get("train_data", "data/train"),
                                max_seq_len=batch_cfg.get("max_seq_len", 4096),
                                vocab_size=model_config.vocab_size)
    # one data shard per data-parallel rank (TP/CP/PP ranks of a replica read the same batch)
    sampler = DistributedSampler(dataset, num_replicas=trainer.dp_size, rank=trainer.dp_rank)
    loader = DataLoader(dataset, batch_size=batch_cfg.get("micro_batch_size", 4), sampler=sampler,
                        collate_fn=TextCollator(),
                        num_workers=data_cfg.get("num_workers", 4),
                        pin_memory=torch.cuda.is_available())
    start = 0
    resume_from = resolve_resume(resume_from, tcfg, trainer.ckpt_mgr)
    if resume_from:
        extra = trainer.ckpt_mgr.load(trainer.model, trainer.optimizer, trainer.scheduler,
                                      resume_from, sampler=sampler)
        start = int(extra.get("step", 0))
    total = max_steps or (tcfg.get("scheduler", {}) or {}).get("total_steps", 100000)
    trainer.train(loader, total, start, sampler)
    return trainer
