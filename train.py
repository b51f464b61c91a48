"""Training entry point, launched under torchrun (one process per GPU).

    torchrun --standalone --nproc_per_node=8 train.py --config config/llama2_7b_2d.yaml --tp-size 2
    torchrun --standalone --nproc_per_node=4 train.py --config config/test_tiny.yaml --tp-size 2 --backend gloo

Flags and their meaning are the reference's (``train.py:38-79``); ``--max-steps``
also moves the schedule's end.  ``--resume-from`` accepts a checkpoint
directory or a run directory (newest valid checkpoint).
"""

from __future__ import annotations

import argparse

from build_your_own_distributed_training_b200.config import TrainingConfig
from build_your_own_distributed_training_b200.parallel.process_groups import destroy_distributed
from build_your_own_distributed_training_b200.training.trainer import Trainer


def parse_args(argv: list[str] | None = None) -> argparse.Namespace:
    p = argparse.ArgumentParser(description="2-D parallel (ZeRO-3 x TP) LLaMA training.")
    p.add_argument("--config", type=str, required=True, help="YAML config path.")
    p.add_argument("--tp-size", type=int, default=None)
    p.add_argument("--dp-size", type=int, default=None)
    p.add_argument("--backend", type=str, default=None, help="nccl | gloo")
    p.add_argument("--run-id", type=str, default=None)
    p.add_argument("--resume-from", type=str, default=None)
    p.add_argument("--max-steps", type=int, default=None)
    p.add_argument("--gpu-type", type=str, default="b200", help="peak-FLOPs key for MFU")
    return p.parse_args(argv)


def build_config(args: argparse.Namespace) -> TrainingConfig:
    cfg = TrainingConfig.from_yaml(args.config)
    if args.tp_size is not None:
        cfg.parallel.tp_size = args.tp_size
    if args.dp_size is not None:
        cfg.parallel.dp_size = args.dp_size
    if args.backend is not None:
        cfg.backend = args.backend
    if args.run_id is not None:
        cfg.run_id = args.run_id
    if args.resume_from is not None:
        cfg.resume_from = args.resume_from
    if args.max_steps is not None:
        cfg.max_steps = args.max_steps
        cfg.scheduler.max_steps = args.max_steps
    return cfg


def main(argv: list[str] | None = None) -> None:
    args = parse_args(argv)
    cfg = build_config(args)
    try:
        Trainer(cfg, gpu_type=args.gpu_type).train()
    finally:
        destroy_distributed()


if __name__ == "__main__":
    main()
