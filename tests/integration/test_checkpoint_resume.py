"""Continuous vs save/resume training is bit-identical (loss and weights)."""

import pytest
import torch

from build_your_own_distributed_training_b200.checkpointing.checkpoint import load_checkpoint, save_checkpoint
from build_your_own_distributed_training_b200.parallel.process_groups import build_process_context
from build_your_own_distributed_training_b200.training.loop import train_step
from build_your_own_distributed_training_b200.training.trainer import Trainer
from tests._dist_utils import run_distributed
from tests.helpers import tiny_config


def _run(rank, world, tp, tmp, full):
    ctx = build_process_context(tp, backend="gloo", verbose=False)

    def mk():
        cfg = tiny_config(tmp, parallel__tp_size=tp, run_id="resume")
        return cfg, Trainer(cfg, ctx=ctx, gpu_type="cpu")

    cfg, a = mk()
    losses_a = []
    for s in range(8):
        w, _ = a._next_window()
        losses_a.append(train_step(a.model, w, a.optimizer, a.scheduler, ctx, cfg, gpu_type="cpu").loss)
        a.step += 1
        if s == 3:
            path = save_checkpoint(a.model, a.optimizer, a.scheduler, a.step, cfg, ctx, full=full)
    final_a = [u.master.clone() for u in a.model.units]
    cfg, b = mk()
    b.step = load_checkpoint(b.model, b.optimizer, b.scheduler, path, ctx)
    b._fast_forward_data(b.step)
    losses_b = []
    for _ in range(4):
        w, _ = b._next_window()
        losses_b.append(train_step(b.model, w, b.optimizer, b.scheduler, ctx, cfg, gpu_type="cpu").loss)
    assert losses_b == losses_a[4:], (losses_a, losses_b)
    for x, y in zip(final_a, [u.master for u in b.model.units]):
        assert torch.equal(x, y)
    assert a.scheduler.get_last_lr() == b.scheduler.get_last_lr()


@pytest.mark.parametrize("world,tp,full", [(1, 1, False), (2, 1, False), (4, 2, False), (4, 2, True)])
def test_resume_is_bit_exact(tmp_path, world, tp, full):
    run_distributed(_run, world, tp, str(tmp_path), full)


def _save_at(rank, world, tp, tmp):
    ctx = build_process_context(tp, backend="gloo", verbose=False)
    cfg = tiny_config(tmp, parallel__tp_size=tp, run_id="topo")
    t = Trainer(cfg, ctx=ctx, gpu_type="cpu")
    w, _ = t._next_window()
    train_step(t.model, w, t.optimizer, t.scheduler, ctx, cfg, gpu_type="cpu")
    save_checkpoint(t.model, t.optimizer, t.scheduler, 1, cfg, ctx, full=False)


def _load_at(rank, world, tp, tmp):
    import glob
    ctx = build_process_context(tp, backend="gloo", verbose=False)
    cfg = tiny_config(tmp, parallel__tp_size=tp, run_id="topo")
    t = Trainer(cfg, ctx=ctx, gpu_type="cpu")
    path = sorted(glob.glob(f"{tmp}/**/step_1", recursive=True))[0]
    with pytest.raises(ValueError, match="topology that wrote them"):
        load_checkpoint(t.model, t.optimizer, t.scheduler, path, ctx)


def test_sharded_load_on_another_topology_fails_early(tmp_path):
    run_distributed(_save_at, 2, 1, str(tmp_path))   # tp1 x dp2
    run_distributed(_load_at, 2, 2, str(tmp_path))   # tp2 x dp1: same world size, other layout
