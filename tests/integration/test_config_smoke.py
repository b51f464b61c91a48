"""Every shipped YAML config trains two steps on CPU ranks.

Each config keeps its parallel layout flags (sharding strategy, sequence
parallelism, loss parallelism, activation checkpointing, accumulation), with
the model shrunk to a few KB and tp capped at 2 so it fits gloo ranks; the
run checks that the loss is finite and that the TP ranks agree on it.
"""
import glob
import math
import os

import pytest

from build_your_own_distributed_training_b200.config import TrainingConfig
from build_your_own_distributed_training_b200.parallel.process_groups import build_process_context
from build_your_own_distributed_training_b200.training.loop import train_step
from build_your_own_distributed_training_b200.training.trainer import Trainer
from tests._dist_utils import run_distributed
from tests.helpers import ROOT

CONFIGS = sorted(glob.glob(os.path.join(ROOT, "config", "*.yaml")))


def _shrunk(path: str, tmp: str) -> TrainingConfig:
    cfg = TrainingConfig.from_yaml(path)
    m = cfg.model
    gqa = m.n_kv_heads is not None and m.n_kv_heads < m.n_heads
    m.vocab_size, m.d_model, m.n_layers, m.n_heads = 256, 64, 2, 4
    m.n_kv_heads = 2 if gqa else 4
    m.ffn_hidden_size, m.max_seq_len = 172, 64
    cfg.data.seq_len, cfg.data.micro_batch_size, cfg.data.global_batch_size = 32, 2, 0
    cfg.data.dataset_path = "uniform" if cfg.data.dataset_path == "uniform" else "synthetic"
    cfg.data.num_workers = 0
    cfg.grad_accum_steps = min(cfg.grad_accum_steps, 2)
    cfg.parallel.tp_size = min(cfg.parallel.tp_size, 2)
    cfg.parallel.dp_size = -1
    cfg.backend = "gloo"
    cfg.checkpoint_dir = tmp
    cfg.eval_interval = cfg.save_interval = cfg.profile_steps = 0
    cfg.log_interval = 10 ** 9
    return cfg


def _run(rank, world, path, tmp):
    cfg = _shrunk(path, tmp)
    ctx = build_process_context(cfg.parallel.tp_size, backend="gloo", verbose=False)
    t = Trainer(cfg, ctx=ctx, gpu_type="cpu")
    losses = []
    for _ in range(2):
        w, _ = t._next_window()
        losses.append(train_step(t.model, w, t.optimizer, t.scheduler, ctx, cfg, gpu_type="cpu").loss)
        t.step += 1
    assert all(math.isfinite(x) for x in losses), losses
    import torch
    import torch.distributed as dist
    if cfg.parallel.tp_size > 1:
        mine = torch.tensor(losses, dtype=torch.float64)
        other = mine.clone()
        dist.all_reduce(other, op=dist.ReduceOp.MAX, group=ctx.tp_group)
        assert torch.equal(mine, other), "TP ranks disagree on the loss"


@pytest.mark.parametrize("path", CONFIGS, ids=[os.path.basename(p)[:-5] for p in CONFIGS])
def test_config_trains_two_steps(tmp_path, path):
    tp = min(TrainingConfig.from_yaml(path).parallel.tp_size, 2)
    run_distributed(_run, 2 * tp, path, str(tmp_path))
