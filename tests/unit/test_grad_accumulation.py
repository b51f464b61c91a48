"""Gradient accumulation: K micro-steps of loss/K equal one step on the K-times batch."""

import torch

from build_your_own_distributed_training_b200.models.transformer import build_model
from tests.helpers import tiny_config


def test_plain_model_accumulation_equals_full_batch():
    cfg = tiny_config()
    torch.manual_seed(0)
    m = build_model(cfg.model)
    toks = torch.randint(0, 256, (4, 17))
    for i in range(2):
        part = toks[2 * i:2 * i + 2]
        (m(part[:, :-1], labels=part[:, 1:])[1] / 2).backward()
    acc = [p.grad.clone() for p in m.parameters()]
    m.zero_grad()
    m(toks[:, :-1], labels=toks[:, 1:])[1].backward()
    for a, p in zip(acc, m.parameters()):
        assert torch.allclose(a, p.grad, atol=1e-6)


def test_loss_over_accum_math():
    losses = [torch.tensor(2.0), torch.tensor(4.0)]
    assert float(sum(l / 2 for l in losses)) == 3.0
