"""Activation checkpointing recomputes each block in backward and changes no number.

Two runs from the same seed, with and without per-block checkpointing, must
produce bit-identical losses and weights (the recompute runs the same ops on
the same inputs).  Runs as one gloo rank and as tp=2 x dp=1.
"""
import pytest
import torch

from build_your_own_distributed_training_b200.parallel.process_groups import build_process_context
from build_your_own_distributed_training_b200.training.loop import train_step
from build_your_own_distributed_training_b200.training.trainer import Trainer
from tests._dist_utils import run_distributed
from tests.helpers import tiny_config


def _run(rank, world, tp):
    ctx = build_process_context(tp, backend="gloo", verbose=False)
    out = []
    for ac in (False, True):
        cfg = tiny_config(None, parallel__tp_size=tp, parallel__activation_checkpointing=ac)
        t = Trainer(cfg, ctx=ctx, gpu_type="cpu")
        assert any(getattr(m, "_ac_wrapped", False) for m in t.model.modules()) == ac
        losses = []
        for _ in range(3):
            w, _ = t._next_window()
            losses.append(train_step(t.model, w, t.optimizer, t.scheduler, ctx, cfg, gpu_type="cpu").loss)
        out.append((losses, [u.master.clone() for u in t.model.units]))
    (la, wa), (lb, wb) = out
    assert la == lb, (la, lb)
    for x, y in zip(wa, wb):
        assert torch.equal(x, y)


@pytest.mark.parametrize("world,tp", [(1, 1), (2, 2)])
def test_checkpointing_is_bit_equal(world, tp):
    run_distributed(_run, world, tp)
