"""Unified command line: ``pretrain | sft | grpo | dpo | eval``.

Same sub-commands and flags as the reference's ``train.py`` (reference:
train.py:36-146), so existing launch scripts work unchanged:

    python train.py pretrain --model-config configs/model/debug.yaml --stage 1
    torchrun --nproc_per_node=8 train.py pretrain --model-config configs/model/large.yaml
    python train.py sft --model-config configs/model/debug.yaml --variant fusion
    python train.py grpo --model-config configs/model/debug.yaml
    python train.py dpo --model-config configs/model/debug.yaml
    python train.py eval --model-config configs/model/debug.yaml --checkpoint ckpt/checkpoint.pt
    python train.py --nproc 8 pretrain --model-config configs/model/small.yaml   # one process per GPU

Differences: ``--stage`` reaches the pretrainer (stage 3 enables YARN
long-context scaling; the reference dropped the flag), ``--max-steps`` caps a
run, and ``eval`` actually runs the named benchmarks (the reference printed
their names only, train.py:143-146) and accepts a DCP checkpoint directory as
well as a ``checkpoint.pt`` file.
"""

from __future__ import annotations

import argparse
import sys
from typing import List, Optional

DEFAULT_TRAINING_CONFIGS = {
    "pretrain": "configs/training/pretrain.yaml",
    "sft": "configs/training/sft.yaml",
    "grpo": "configs/training/rl.yaml",
    "dpo": "configs/training/rl.yaml",
}


def _common(sub: argparse.ArgumentParser) -> None:
    sub.add_argument("--model-config", required=True, help="model config YAML")
    sub.add_argument("--training-config", default=None,
                     help="training config YAML (per-phase default when omitted)")
    sub.add_argument("--resume", default=None, help="checkpoint directory to resume from")
    sub.add_argument("--max-samples", type=int, default=None, help="cap the dataset size")
    sub.add_argument("--max-steps", type=int, default=None, help="cap the number of steps")


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="nano_qwen_b200 training CLI",
                                formatter_class=argparse.RawDescriptionHelpFormatter)
    subs = p.add_subparsers(dest="command", required=True)
    pre = subs.add_parser("pretrain", help="pretraining (stage 1 general, 2 reasoning, 3 long context)")
    _common(pre)
    pre.add_argument("--stage", type=int, default=1, choices=[1, 2, 3])
    sft = subs.add_parser("sft", help="supervised fine-tuning")
    _common(sft)
    sft.add_argument("--variant", default="cold_start", choices=["cold_start", "fusion"])
    _common(subs.add_parser("grpo", help="group relative policy optimisation"))
    _common(subs.add_parser("dpo", help="direct preference optimisation"))
    ev = subs.add_parser("eval", help="evaluation benchmarks")
    ev.add_argument("--model-config", required=True)
    ev.add_argument("--checkpoint", required=True, help="checkpoint.pt file or DCP directory")
    ev.add_argument("--benchmarks", nargs="+", default=["hellaswag", "mmlu"])
    ev.add_argument("--max-samples", type=int, default=None)
    ev.add_argument("--output", default=None, help="write results JSON here")
    return p


def load_model_for_eval(model_config: str, checkpoint: str):
    import torch
    from pathlib import Path

    from .config import ModelConfig
    from .models import Qwen3Model
    cfg = ModelConfig.from_yaml(model_config)
    model = Qwen3Model(cfg)
    ck = Path(checkpoint)
    if ck.is_dir():
        if (ck / "checkpoint.pt").exists():
            ck = ck / "checkpoint.pt"
        else:
            from .training.checkpoint import CheckpointManager
            CheckpointManager(save_dir=str(ck.parent)).load(model, checkpoint_dir=str(ck))
            return model
    state = torch.load(str(ck), map_location="cpu", weights_only=False)
    model.load_state_dict(state["model"] if "model" in state else state)
    return model


def relaunch_argv(argv: List[str]) -> Optional[List[str]]:
    """``--nproc N`` (N > 1) before the sub-command: the command line that
    runs the same sub-command with one process per GPU through
    ``torch.distributed.run`` on this node (what the reference's
    scripts/*.sh wrappers did with torchrun).  None when no relaunch is
    needed (single process, or already inside a distributed launch)."""
    if "--nproc" not in argv:
        return None
    i = argv.index("--nproc")
    n = int(argv[i + 1])
    rest = argv[:i] + argv[i + 2:]
    if n <= 1 or "LOCAL_RANK" in __import__("os").environ:
        return None
    import os
    script = os.path.abspath(sys.argv[0]) if sys.argv and sys.argv[0].endswith(".py") else "train.py"
    return [sys.executable, "-m", "torch.distributed.run", "--standalone", "--nnodes=1",
            f"--nproc-per-node={n}", "--local-addr", "127.0.0.1", script] + rest


def main(argv: Optional[List[str]] = None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    cmd = relaunch_argv(argv)
    if cmd is not None:
        import subprocess
        return subprocess.call(cmd)
    if "--nproc" in argv:  # a single process, or already launched per GPU
        i = argv.index("--nproc")
        argv = argv[:i] + argv[i + 2:]
    args = build_parser().parse_args(argv)
    if args.command != "eval" and args.training_config is None:
        args.training_config = DEFAULT_TRAINING_CONFIGS[args.command]
    if args.command == "pretrain":
        from .training.pretrain import run_pretraining
        run_pretraining(args.model_config, args.training_config, resume_from=args.resume,
                        stage=args.stage, max_steps=args.max_steps)
    elif args.command == "sft":
        from .training.sft import run_sft
        run_sft(args.model_config, args.training_config, variant=args.variant,
                resume_from=args.resume, max_samples=args.max_samples, max_steps=args.max_steps)
    elif args.command == "grpo":
        from .training.grpo import run_grpo
        run_grpo(args.model_config, args.training_config, resume_from=args.resume,
                 max_samples=args.max_samples, max_steps=args.max_steps)
    elif args.command == "dpo":
        from .training.dpo import run_dpo
        run_dpo(args.model_config, args.training_config, resume_from=args.resume,
                max_samples=args.max_samples, max_steps=args.max_steps)
    elif args.command == "eval":
        import torch

        from .data.tokenizer import Tokenizer
        from .eval.benchmarks import STANDARD_BENCHMARKS, BenchmarkRunner
        from .eval.evaluate import Evaluator
        device = torch.device("cuda" if torch.cuda.is_available() else "cpu")
        model = load_model_for_eval(args.model_config, args.checkpoint).to(device).eval()
        if device.type == "cuda":
            from .training.optimizer import attach_param_store
            attach_param_store(model)
        runner = BenchmarkRunner(Evaluator(model, Tokenizer(), device=device))
        print(f"Running benchmarks: {args.benchmarks}")
        for name in args.benchmarks:
            spec = STANDARD_BENCHMARKS.get(name, {"type": "multiple_choice",
                                                  "data_path": f"benchmarks/{name}.jsonl"})
            runner.run_benchmark(name, spec["data_path"], spec["type"], args.max_samples)
        if args.output:
            runner.save_results(args.output)
    return 0


if __name__ == "__main__":
    sys.exit(main())
