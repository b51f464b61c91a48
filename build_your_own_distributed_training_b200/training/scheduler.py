"""Linear warmup then cosine decay to ``min_lr`` as a ``LambdaLR`` multiplier.

Same curve and checks as ``src/training/scheduler.py:40-111``: warmup
``(step+1)/warmup``; cosine from 1 to ``min_lr/peak`` over
``[warmup, max_steps]``; constant afterwards.
"""

from __future__ import annotations

import math
from collections.abc import Callable

import torch
from torch.optim.lr_scheduler import LambdaLR


def lr_lambda_factory(peak_lr: float, warmup_steps: int, max_steps: int,
                      min_lr: float) -> Callable[[int], float]:
    if max_steps <= warmup_steps:
        raise ValueError(f"max_steps({max_steps}) must exceed warmup_steps({warmup_steps}).")
    if min_lr > peak_lr:
        raise ValueError(f"min_lr({min_lr}) must be <= peak_lr({peak_lr}).")
    floor = min_lr / peak_lr if peak_lr > 0 else 0.0
    span = max(1, max_steps - warmup_steps)

    def fn(step: int) -> float:
        if step < warmup_steps:
            return (step + 1) / max(1, warmup_steps)
        if step >= max_steps:
            return floor
        frac = (step - warmup_steps) / span
        return floor + (1.0 - floor) * 0.5 * (1.0 + math.cos(math.pi * frac))

    return fn


def build_scheduler(optimizer: torch.optim.Optimizer, cfg, peak_lr: float) -> LambdaLR:
    return LambdaLR(optimizer, lr_lambda_factory(peak_lr, cfg.warmup_steps, cfg.max_steps, cfg.min_lr))
