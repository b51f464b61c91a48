"""Failures injected on the host: crash during save, a rank that raises, NaN gradients.

No GPU is faulted, trapped or hung: every failure is a host exception, a
dropped file, or a NaN written into host data before the step.
"""

import os
import time

import pytest
import torch
import torch.distributed as dist

from build_your_own_distributed_training_b200.checkpointing.checkpoint import save_checkpoint
from build_your_own_distributed_training_b200.checkpointing.recovery import find_latest_valid_checkpoint
from build_your_own_distributed_training_b200.parallel.process_groups import build_process_context
from build_your_own_distributed_training_b200.training.grad_utils import GradNotFiniteError
from build_your_own_distributed_training_b200.training.loop import train_step
from build_your_own_distributed_training_b200.training.trainer import Trainer
from tests._dist_utils import run_distributed
from tests.helpers import tiny_config


def _crash_mid_save(rank, world, tmp):
    cfg = tiny_config(tmp, run_id="crash")
    ctx = build_process_context(1, backend="gloo", verbose=False)
    tr = Trainer(cfg, ctx=ctx, gpu_type="cpu")
    for s in range(1, 13):
        w, _ = tr._next_window()
        train_step(tr.model, w, tr.optimizer, tr.scheduler, ctx, cfg, gpu_type="cpu")
        tr.step = s
        if s in (5, 10):
            save_checkpoint(tr.model, tr.optimizer, tr.scheduler, s, cfg, ctx)
    # "crash" while writing step 12: shards on disk, marker never written
    d = save_checkpoint(tr.model, tr.optimizer, tr.scheduler, 12, cfg, ctx)
    ctx.barrier()
    if rank == 0:
        os.remove(os.path.join(d, "_SUCCESS"))
    ctx.barrier()
    run_dir = os.path.dirname(d)
    assert find_latest_valid_checkpoint(run_dir) == os.path.join(run_dir, "step_10")
    # resume from the run directory: the newest valid checkpoint is picked
    cfg2 = tiny_config(tmp, run_id="crash", resume_from=run_dir)
    tr2 = Trainer(cfg2, ctx=ctx, gpu_type="cpu")
    assert tr2.step == 10
    w, _ = tr2._next_window()
    m = train_step(tr2.model, w, tr2.optimizer, tr2.scheduler, ctx, cfg2, gpu_type="cpu")
    assert m.loss == m.loss  # finite, training continues


def test_crash_mid_save_recovers_from_previous(tmp_path):
    run_distributed(_crash_mid_save, 2, str(tmp_path))


def _nan_on_one_rank(rank, world):
    cfg = tiny_config()
    ctx = build_process_context(1, backend="gloo", verbose=False)
    tr = Trainer(cfg, ctx=ctx, gpu_type="cpu")
    before = [u.master.clone() for u in tr.model.units]
    w, _ = tr._next_window()
    if rank == 1:  # poison one embedding row that this batch uses
        tok = int(w[0]["input_ids"][0, 0])
        with torch.no_grad():
            for u in tr.model.units:
                for e in u.entries:
                    if e.fqn == "tok_embeddings.weight":
                        e.param.view(-1, 64)[tok].fill_(float("nan"))
    with pytest.raises(GradNotFiniteError):
        train_step(tr.model, w, tr.optimizer, tr.scheduler, ctx, cfg, gpu_type="cpu")
    # the update was skipped on every rank
    for a, u in zip(before, tr.model.units):
        assert torch.equal(a, u.master)
    assert tr.scheduler.last_epoch == 0


def test_nan_on_one_rank_raises_on_all_and_skips_update():
    run_distributed(_nan_on_one_rank, 2)


def _rank_raises(rank, world):
    os.environ["DTB_PG_TIMEOUT_S"] = "20"
    cfg = tiny_config()
    ctx = build_process_context(1, backend="gloo", verbose=False)
    tr = Trainer(cfg, ctx=ctx, gpu_type="cpu")
    if rank == 1:
        raise RuntimeError("injected failure on rank 1")
    t0 = time.time()
    with pytest.raises(Exception):
        for _ in range(3):
            w, _ = tr._next_window()
            train_step(tr.model, w, tr.optimizer, tr.scheduler, ctx, cfg, gpu_type="cpu")
    assert time.time() - t0 < 110  # the survivor errors out instead of hanging
    raise SystemExit(0)


def test_rank_that_raises_does_not_hang_the_others():
    with pytest.raises(Exception, match="injected failure on rank 1"):
        run_distributed(_rank_raises, 2)
