"""End-to-end learning on the Markov corpus (the reference's convergence obligation)."""

import pytest

from build_your_own_distributed_training_b200.parallel.process_groups import build_process_context
from build_your_own_distributed_training_b200.training.loop import train_step
from build_your_own_distributed_training_b200.training.trainer import Trainer
from tests._dist_utils import run_distributed
from tests.helpers import tiny_config


def _train(rank, world, tp, steps, strategy):
    cfg = tiny_config(parallel__tp_size=tp, max_steps=steps, parallel__sharding_strategy=strategy)
    cfg.scheduler.max_steps = steps
    ctx = build_process_context(tp, backend="gloo", verbose=False)
    tr = Trainer(cfg, ctx=ctx, gpu_type="cpu")
    losses = []
    for _ in range(steps):
        w, _ = tr._next_window()
        losses.append(train_step(tr.model, w, tr.optimizer, tr.scheduler, ctx, cfg, gpu_type="cpu").loss)
    first, last = sum(losses[:3]) / 3, sum(losses[-3:]) / 3
    assert last < first - 1.0, (first, last)


@pytest.mark.parametrize("world,tp,strategy", [(1, 1, "FULL_SHARD"), (2, 1, "FULL_SHARD"), (2, 2, "FULL_SHARD"),
                                               (4, 2, "FULL_SHARD"), (2, 1, "NO_SHARD")])
def test_tiny_converges(world, tp, strategy):
    run_distributed(_train, world, tp, 60, strategy)
