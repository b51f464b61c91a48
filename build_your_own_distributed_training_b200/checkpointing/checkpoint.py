"""Atomic sharded checkpoints.

Layout, file names, meta schema and marker protocol are the reference's
(``src/checkpointing/checkpoint.py:9-227``)::

    {checkpoint_dir}/{run_id}/step_{N}/
        meta.json         step, world_size, tp_size, dp_size, format, config   (rank 0)
        scheduler.pt      LambdaLR state                                        (rank 0)
        rank_{r}/model.pt optim.pt rng.pt                                       (every rank)
        model_full.pt optim_full.pt                                             (full format, rank 0)
        _SUCCESS          text: the step, written last

Every file is written to ``*.tmp`` then renamed; text files are fsync'd.
Barrier, marker, barrier: a step directory with ``_SUCCESS`` is complete.
Loads use ``torch.load(weights_only=True)`` (all our files qualify; files from
older writers that need pickle fall back to ``weights_only=False``), which
fixes the reference's resume failing on its own ``rng.pt`` under torch >= 2.6.
"""

from __future__ import annotations

import json
import os
import pickle
from typing import Any

import torch

from ..parallel.state_dict import (get_model_state_dict, get_optimizer_state_dict,
                                   load_model_state_dict, load_optimizer_state_dict)
from ..utils.seed import get_rng_state, set_rng_state

SUCCESS_MARKER = "_SUCCESS"
META_FILE = "meta.json"
SCHEDULER_FILE = "scheduler.pt"


def _atomic_torch_save(obj: Any, path: str) -> None:
    tmp = path + ".tmp"
    torch.save(obj, tmp)
    os.replace(tmp, path)


def _atomic_write_text(text: str, path: str) -> None:
    tmp = path + ".tmp"
    with open(tmp, "w") as f:
        f.write(text)
        f.flush()
        os.fsync(f.fileno())
    os.replace(tmp, path)


def safe_load(path: str) -> Any:
    """``torch.load`` on CPU with ``weights_only=True``, pickle fallback for legacy files."""
    try:
        return torch.load(path, map_location="cpu", weights_only=True)
    except pickle.UnpicklingError:
        return torch.load(path, map_location="cpu", weights_only=False)


def checkpoint_path(config: Any, step: int) -> str:
    return os.path.join(config.checkpoint_dir, config.run_id, f"step_{step}")


def save_checkpoint(model: Any, optimizer: torch.optim.Optimizer, scheduler: Any, step: int,
                    config: Any, ctx: Any, *, full: bool = False) -> str:
    d = checkpoint_path(config, step)
    rank_dir = os.path.join(d, f"rank_{ctx.rank}")
    os.makedirs(rank_dir, exist_ok=True)
    msd = get_model_state_dict(model, full=full)
    osd = get_optimizer_state_dict(model, optimizer, full=full)
    if full:
        if ctx.is_rank0:
            _atomic_torch_save(msd, os.path.join(d, "model_full.pt"))
            _atomic_torch_save(osd, os.path.join(d, "optim_full.pt"))
    else:
        _atomic_torch_save(msd, os.path.join(rank_dir, "model.pt"))
        _atomic_torch_save(osd, os.path.join(rank_dir, "optim.pt"))
    _atomic_torch_save(get_rng_state(), os.path.join(rank_dir, "rng.pt"))
    if ctx.is_rank0:
        _atomic_torch_save(scheduler.state_dict(), os.path.join(d, SCHEDULER_FILE))
        meta = {"step": step, "world_size": ctx.world_size, "tp_size": ctx.dims.tp_size,
                "dp_size": ctx.dims.dp_size, "format": "full" if full else "sharded",
                "config": config.to_dict()}
        _atomic_write_text(json.dumps(meta, indent=2), os.path.join(d, META_FILE))
    ctx.barrier()
    if ctx.is_rank0:
        _atomic_write_text(str(step), os.path.join(d, SUCCESS_MARKER))
    ctx.barrier()
    return d


def load_checkpoint(model: Any, optimizer: torch.optim.Optimizer, scheduler: Any, path: str,
                    ctx: Any, *, full: bool | None = None, restore_rng: bool = True) -> int:
    """Restore model, optimizer, scheduler and RNG; returns the saved step.

    ``full=None`` picks the format recorded in ``meta.json``.
    """
    if not os.path.exists(os.path.join(path, SUCCESS_MARKER)):
        raise FileNotFoundError(
            f"[rank {ctx.rank}] checkpoint {path} has no {SUCCESS_MARKER} marker: it is "
            "incomplete or corrupt; refusing to load.")
    with open(os.path.join(path, META_FILE)) as f:
        meta = json.load(f)
    if full is None:
        full = meta.get("format") == "full"
    if not full:
        saved = (meta.get("world_size"), meta.get("tp_size"), meta.get("dp_size"))
        now = (ctx.world_size, ctx.dims.tp_size, ctx.dims.dp_size)
        if saved != now:
            raise ValueError(
                f"[rank {ctx.rank}] sharded checkpoint {path} was written by world_size={saved[0]} "
                f"(tp={saved[1]}, dp={saved[2]}) but this run is world_size={now[0]} (tp={now[1]}, "
                f"dp={now[2]}): shards are only valid on the topology that wrote them; resume with "
                "that topology or save/load the full format.")
    rank_dir = os.path.join(path, f"rank_{ctx.rank}")
    if full:
        load_model_state_dict(model, safe_load(os.path.join(path, "model_full.pt")), full=True)
        load_optimizer_state_dict(model, optimizer, safe_load(os.path.join(path, "optim_full.pt")),
                                  full=True)
    else:
        mfile = os.path.join(rank_dir, "model.pt")
        if not os.path.exists(mfile):
            raise FileNotFoundError(
                f"[rank {ctx.rank}] missing shard {mfile}: the checkpoint was saved with another "
                "world size; resume on the saving topology or load a full-format checkpoint.")
        load_model_state_dict(model, safe_load(mfile), full=False)
        load_optimizer_state_dict(model, optimizer, safe_load(os.path.join(rank_dir, "optim.pt")),
                                  full=False)
    scheduler.load_state_dict(safe_load(os.path.join(path, SCHEDULER_FILE)))
    if restore_rng and os.path.exists(os.path.join(rank_dir, "rng.pt")):
        set_rng_state(safe_load(os.path.join(rank_dir, "rng.pt")))
    return int(meta["step"])
