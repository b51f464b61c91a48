"""Small builders shared by the CPU tests."""

from __future__ import annotations

import os

from build_your_own_distributed_training_b200.config import TrainingConfig

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TINY = os.path.join(ROOT, "config", "test_tiny.yaml")


def tiny_config(tmpdir: str | None = None, **over) -> TrainingConfig:
    cfg = TrainingConfig.from_yaml(TINY)
    cfg.eval_interval = 0
    cfg.save_interval = 0
    cfg.log_interval = 10 ** 9
    if tmpdir is not None:
        cfg.checkpoint_dir = tmpdir
    for k, v in over.items():
        obj = cfg
        parts = k.split("__")
        for p in parts[:-1]:
            obj = getattr(obj, p)
        setattr(obj, parts[-1], v)
    return cfg
