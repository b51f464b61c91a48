import math

import pytest
import torch

from build_your_own_distributed_training_b200.config import SchedulerConfig
from build_your_own_distributed_training_b200.training.scheduler import build_scheduler, lr_lambda_factory


def test_warmup_is_linear_and_monotone():
    f = lr_lambda_factory(1e-3, 10, 100, 1e-4)
    vals = [f(s) for s in range(10)]
    assert vals == sorted(vals) and abs(vals[0] - 0.1) < 1e-12 and abs(vals[-1] - 1.0) < 1e-12


def test_cosine_and_floor():
    f = lr_lambda_factory(1e-3, 10, 110, 1e-4)
    mid = f(60)
    assert abs(mid - (0.1 + 0.9 * 0.5 * (1 + math.cos(math.pi * 0.5)))) < 1e-12
    assert abs(f(110) - 0.1) < 1e-12 and abs(f(500) - 0.1) < 1e-12


def test_bad_args():
    with pytest.raises(ValueError):
        lr_lambda_factory(1e-3, 10, 10, 0)
    with pytest.raises(ValueError):
        lr_lambda_factory(1e-3, 1, 10, 1e-2)


def test_resume_lr_equality():
    p = torch.nn.Parameter(torch.zeros(1))
    cfg = SchedulerConfig(warmup_steps=5, max_steps=50, min_lr=1e-4)
    o1 = torch.optim.AdamW([p], lr=1e-3)
    s1 = build_scheduler(o1, cfg, 1e-3)
    for _ in range(17):
        o1.step()
        s1.step()
    o2 = torch.optim.AdamW([p], lr=1e-3)
    s2 = build_scheduler(o2, cfg, 1e-3)
    s2.load_state_dict(s1.state_dict())
    assert s2.get_last_lr() == s1.get_last_lr()
