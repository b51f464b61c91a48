"""File-level fault injection against the checkpoint validator."""

import json
import os

import pytest

from build_your_own_distributed_training_b200.checkpointing.checkpoint import save_checkpoint
from build_your_own_distributed_training_b200.checkpointing.recovery import (CheckpointValidationError,
                                                                             find_latest_valid_checkpoint,
                                                                             require_valid_checkpoint,
                                                                             validate_checkpoint)
from build_your_own_distributed_training_b200.parallel.process_groups import build_process_context
from build_your_own_distributed_training_b200.training.trainer import Trainer
from tests.helpers import tiny_config


@pytest.fixture()
def saved(tmp_path, single_process_pg):
    cfg = tiny_config(str(tmp_path), run_id="corrupt")
    ctx = build_process_context(1, backend="gloo", verbose=False)
    tr = Trainer(cfg, ctx=ctx, gpu_type="cpu")
    paths = [save_checkpoint(tr.model, tr.optimizer, tr.scheduler, s, cfg, ctx) for s in (5, 10)]
    return cfg, paths


def test_valid_checkpoint_passes_deep_check(saved):
    cfg, paths = saved
    res = require_valid_checkpoint(paths[-1], expected_config=cfg.to_dict(), deep=True)
    assert res.step == 10 and res.world_size == 1


def test_missing_rank_shard_via_meta(saved):
    _, paths = saved
    meta = os.path.join(paths[-1], "meta.json")
    m = json.load(open(meta))
    m["world_size"] = 2
    json.dump(m, open(meta, "w"))
    res = validate_checkpoint(paths[-1])
    assert not res.is_valid and any("rank 1" in e for e in res.errors)


def test_truncated_shard(saved):
    _, paths = saved
    f = os.path.join(paths[-1], "rank_0", "model.pt")
    open(f, "wb").close()
    assert not validate_checkpoint(paths[-1]).is_valid
    with open(f, "wb") as fh:
        fh.write(b"not a checkpoint")
    assert validate_checkpoint(paths[-1], deep=False).is_valid
    assert not validate_checkpoint(paths[-1], deep=True).is_valid


def test_config_mismatch(saved):
    cfg, paths = saved
    other = cfg.to_dict()
    other["model"]["d_model"] = 128
    res = validate_checkpoint(paths[-1], expected_config=other)
    assert not res.is_valid and any("d_model" in e for e in res.errors)
    with pytest.raises(CheckpointValidationError):
        require_valid_checkpoint(paths[-1], expected_config=other)


def test_latest_skips_incomplete(saved):
    _, paths = saved
    os.remove(os.path.join(paths[-1], "_SUCCESS"))
    assert find_latest_valid_checkpoint(os.path.dirname(paths[-1])) == paths[0]
