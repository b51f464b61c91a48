"""Model / optimizer state dicts for the sharding engine.

Keys are the model's parameter FQNs (``tok_embeddings.weight``,
``layers.{i}.attention.wq.weight``, ... ``lm_head.weight``; a tied head is
saved under both names), as with the reference's FSDP state dicts
(``src/parallelism/fsdp_utils.py:230-378``).

Sharded form (one dict per rank): every parameter is split into even dim-0
chunks over the shard (dp) group, on top of its tensor-parallel split, and
this rank stores its chunk as a plain fp32 tensor.  A ``__layout__`` entry
records, per key, the TP split (``row``/``col``/``rep``), the TP-local shape
and the chunk's row range, which is what the reference's DTensor values
encoded.  Optimizer state uses the same keys:
``{"state": {fqn: {"step", "exp_avg", "exp_avg_sq"}}, "param_groups": [...]}``.
Everything is tensors, ints, floats and strings, so the files load with
``torch.load(weights_only=True)``.

Full form: rank 0 receives complete (TP-gathered, dp-gathered) fp32 tensors;
loading it works at any topology.
"""

from __future__ import annotations

from typing import Any

import torch
import torch.distributed as dist
import torch.nn as nn

from .fsdp import FlatUnit, FullyShardedModel


def _chunk_rows(rows: int, world: int, rank: int) -> tuple[int, int]:
    per = -(-rows // world) if rows else 0
    lo = min(rows, rank * per)
    return lo, min(rows, lo + per)


def _aliases(model: FullyShardedModel) -> dict[int, list[str]]:
    names: dict[int, list[str]] = {}
    for n, p in model.module.named_parameters(remove_duplicate=False):
        names.setdefault(id(p), []).append(n)
    return names


def _flat_full(model: FullyShardedModel, u: FlatUnit, shard: torch.Tensor) -> torch.Tensor:
    if model.shard_world == 1:
        return shard.detach().float().clone()
    out = torch.empty(u.numel, dtype=torch.float32, device=shard.device)
    src = shard.detach().float().contiguous()
    if src.is_cuda:
        dist.all_gather_into_tensor(out, src, group=model.comm.group)
    else:
        dist.all_gather(list(out.chunk(model.shard_world)), src, group=model.comm.group)
    return out


def _tp_gather(t: torch.Tensor, kind: str, model: FullyShardedModel) -> torch.Tensor:
    if kind == "rep" or model.tp_size == 1:
        return t
    parts = [torch.empty_like(t) for _ in range(model.tp_size)]
    dist.all_gather(parts, t.contiguous(), group=model.tp_group)
    return torch.cat(parts, dim=0 if kind == "row" else 1)


def _unit_entries(model: FullyShardedModel, flat_shards: dict[str, list[torch.Tensor]], *, full: bool
                  ) -> tuple[dict[str, dict[str, torch.Tensor]], dict[str, Any]]:
    aliases = _aliases(model)
    out: dict[str, dict[str, torch.Tensor]] = {k: {} for k in flat_shards}
    layout: dict[str, Any] = {}
    W, R = model.shard_world, model.shard_rank
    for ui, u in enumerate(model.units):
        fulls = {k: _flat_full(model, u, v[ui]) for k, v in flat_shards.items()}
        for e in u.entries:
            names = aliases.get(id(e.param), [e.fqn])
            for k, flat in fulls.items():
                local = flat[e.offset:e.offset + e.numel].view(e.shape)
                if full:
                    val = _tp_gather(local, e.tp_kind, model).detach().cpu().clone()
                else:
                    lo, hi = _chunk_rows(e.shape[0], W, R)
                    val = local[lo:hi].detach().cpu().clone()
                for n in names:
                    out[k][n] = val
            if not full:
                lo, hi = _chunk_rows(e.shape[0], W, R)
                for n in names:
                    layout[n] = {"tp": e.tp_kind, "local_shape": list(e.shape), "rows": [lo, hi],
                                 "dp_world": W, "dp_rank": R, "tp_size": model.tp_size,
                                 "tp_rank": model.ctx.dims.tp_rank if model.ctx else 0}
    return out, layout


def get_model_state_dict(model: nn.Module, *, full: bool) -> dict[str, Any]:
    if not isinstance(model, FullyShardedModel):
        return model.state_dict()
    vals, layout = _unit_entries(model, {"p": [u.master for u in model.units]}, full=full)
    sd: dict[str, Any] = dict(vals["p"])
    if full:
        rank0 = not dist.is_initialized() or dist.get_rank() == 0
        return sd if rank0 else {}
    sd["__layout__"] = layout
    return sd


def _scatter_into_units(model: FullyShardedModel, values: dict[str, torch.Tensor], *, full: bool,
                        targets: list[torch.Tensor]) -> None:
    """Write per-FQN values (chunks or full tensors) back into per-unit flat shards."""
    W, R = model.shard_world, model.shard_rank
    tpr = model.ctx.dims.tp_rank if model.ctx else 0
    for ui, u in enumerate(model.units):
        dev = targets[ui].device
        flat = torch.zeros(u.numel, dtype=torch.float32, device=dev)
        for e in u.entries:
            if e.fqn not in values:
                raise KeyError(f"state dict is missing {e.fqn!r}")
            v = values[e.fqn].to(dev, torch.float32)
            seg = flat[e.offset:e.offset + e.numel].view(e.shape)
            if full:
                if e.tp_kind == "row":
                    n = e.shape[0]
                    v = v[tpr * n:(tpr + 1) * n]
                elif e.tp_kind == "col":
                    n = e.shape[1]
                    v = v[:, tpr * n:(tpr + 1) * n]
                if tuple(v.shape) != tuple(e.shape):
                    raise ValueError(f"{e.fqn}: shape {tuple(v.shape)} != expected {tuple(e.shape)}")
                seg.copy_(v)
            else:
                lo, hi = _chunk_rows(e.shape[0], W, R)
                if v.shape[0] != hi - lo:
                    raise ValueError(f"{e.fqn}: chunk has {v.shape[0]} rows, expected {hi - lo}; the "
                                     "checkpoint was saved with another topology")
                seg[lo:hi].copy_(v)
        if not full and W > 1:
            dist.all_reduce(flat, group=model.comm.group)
        lo, hi = u.shard_range(R)
        targets[ui].copy_(flat[lo:hi].to(targets[ui].dtype))


def load_model_state_dict(model: nn.Module, state_dict: dict[str, Any], *, full: bool) -> None:
    if not isinstance(model, FullyShardedModel):
        model.load_state_dict(state_dict)
        return
    values = {k: v for k, v in state_dict.items() if k != "__layout__"}
    _scatter_into_units(model, values, full=full, targets=[u.master for u in model.units])
    for u in model.units:
        u.param_shard.copy_(u.master.to(u.param_shard.dtype))
    model.after_optimizer_step()


def get_optimizer_state_dict(model: nn.Module, optimizer: torch.optim.Optimizer, *, full: bool
                             ) -> dict[str, Any]:
    if not isinstance(model, FullyShardedModel):
        return optimizer.state_dict()
    states = [optimizer.state.get(u.master, {}) for u in model.units]
    if not all(states):
        flat = {"exp_avg": [torch.zeros_like(u.master) for u in model.units],
                "exp_avg_sq": [torch.zeros_like(u.master) for u in model.units]}
        steps = [0.0] * len(model.units)
    else:
        flat = {"exp_avg": [s["exp_avg"] for s in states], "exp_avg_sq": [s["exp_avg_sq"] for s in states]}
        steps = [float(s["step"]) for s in states]
    vals, layout = _unit_entries(model, flat, full=full)
    unit_of = {e.fqn: ui for ui, u in enumerate(model.units) for e in u.entries}
    aliases = _aliases(model)
    for ui, u in enumerate(model.units):
        for e in u.entries:
            for n in aliases.get(id(e.param), [e.fqn]):
                unit_of[n] = ui
    state = {n: {"step": torch.tensor(steps[unit_of[n]]), "exp_avg": vals["exp_avg"][n],
                 "exp_avg_sq": vals["exp_avg_sq"][n]} for n in vals["exp_avg"]}
    groups = [{k: (list(v) if isinstance(v, tuple) else v) for k, v in g.items() if k != "params"}
              for g in optimizer.param_groups]
    out: dict[str, Any] = {"state": state, "param_groups": groups}
    if full:
        rank0 = not dist.is_initialized() or dist.get_rank() == 0
        return out if rank0 else {}
    out["__layout__"] = layout
    return out


def load_optimizer_state_dict(model: nn.Module, optimizer: torch.optim.Optimizer,
                              osd: dict[str, Any], *, full: bool) -> None:
    if isinstance(osd, dict) and osd.get("__fsdp_per_rank__"):
        optimizer.load_state_dict(osd["state"])
        return
    if not isinstance(model, FullyShardedModel):
        optimizer.load_state_dict(osd)
        return
    st = osd["state"]
    for key in ("exp_avg", "exp_avg_sq"):
        targets = []
        for u in model.units:
            s = optimizer.state[u.master]
            if key not in s:
                s["exp_avg"] = torch.zeros_like(u.master)
                s["exp_avg_sq"] = torch.zeros_like(u.master)
            targets.append(s[key])
        _scatter_into_units(model, {k: v[key] for k, v in st.items()}, full=full, targets=targets)
    for u in model.units:
        first = u.entries[0].fqn if u.entries else None
        step = float(st[first]["step"]) if first in st else 0.0
        optimizer.state[u.master]["step"] = torch.tensor(step, dtype=torch.float32)
    for g, saved in zip(optimizer.param_groups, osd.get("param_groups", [])):
        for k, v in saved.items():
            g[k] = tuple(v) if k == "betas" else v
