"""Model / optimizer state dicts for the sharding engine.

Keys are the model's parameter FQNs (``tok_embeddings.weight``,
``layers.{i}.attention.wq.weight``, ... ``lm_head.weight``; a tied head is
saved under both names), as with the reference's FSDP state dicts
(``src/parallelism/fsdp_utils.py:230-378``).

Sharded form (one dict per rank): each rank writes exactly the fp32 values
it owns, with no communication.  The engine shards a block's flat buffer into
contiguous ranges, so a rank's piece of a parameter is a contiguous range of
that parameter's flattened (TP-local) values; it is stored as a 1-D fp32
tensor (empty where the rank owns none of it).  A ``__layout__`` entry
records, per key, the TP split (``row``/``col``/``rep``), the TP-local shape
and the flat range ``[lo, hi)``, which is what the reference's DTensor values
encoded.  Loading reads the same ranges back, so a sharded checkpoint resumes
on the topology that wrote it (the loader checks ``meta.json`` first).  Optimizer state uses the same keys:
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


def _local_piece(u: FlatUnit, e: Any, rank: int) -> tuple[int, int, int]:
    """(lo, hi, shard_offset): the range [lo, hi) of entry ``e``'s flattened values that
    lies in ``rank``'s shard of unit ``u``, and where it starts inside that shard."""
    s_lo, s_hi = u.shard_range(rank)
    a, b = max(e.offset, s_lo), min(e.offset + e.numel, s_hi)
    if b <= a:
        return 0, 0, 0
    return a - e.offset, b - e.offset, a - s_lo


def _unit_entries(model: FullyShardedModel, flat_shards: dict[str, list[torch.Tensor]], *, full: bool
                  ) -> tuple[dict[str, dict[str, torch.Tensor]], dict[str, Any]]:
    aliases = _aliases(model)
    out: dict[str, dict[str, torch.Tensor]] = {k: {} for k in flat_shards}
    layout: dict[str, Any] = {}
    W, R = model.shard_world, model.shard_rank
    tpr = model.ctx.dims.tp_rank if model.ctx else 0
    for ui, u in enumerate(model.units):
        if full:
            fulls = {k: _flat_full(model, u, v[ui]) for k, v in flat_shards.items()}
        for e in u.entries:
            names = aliases.get(id(e.param), [e.fqn])
            if full:
                for k, flat in fulls.items():
                    local = flat[e.offset:e.offset + e.numel].view(e.shape)
                    val = _tp_gather(local, e.tp_kind, model).detach().cpu().clone()
                    for n in names:
                        out[k][n] = val
                continue
            lo, hi, so = _local_piece(u, e, R)
            for k, shards in flat_shards.items():
                val = shards[ui].detach()[so:so + (hi - lo)].float().cpu().clone()
                for n in names:
                    out[k][n] = val
            for n in names:
                layout[n] = {"tp": e.tp_kind, "local_shape": list(e.shape), "flat": [lo, hi],
                             "dp_world": W, "dp_rank": R, "tp_size": model.tp_size, "tp_rank": tpr}
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
    """Write per-FQN values back into per-unit flat shards: complete tensors (full form, any
    topology, each rank keeps its TP slice and flat range) or this rank's own flat ranges
    (sharded form, no communication)."""
    R = model.shard_rank
    tpr = model.ctx.dims.tp_rank if model.ctx else 0
    for ui, u in enumerate(model.units):
        dev = targets[ui].device
        s_lo, s_hi = u.shard_range(R)
        shard = torch.zeros(s_hi - s_lo, dtype=torch.float32, device=dev)
        for e in u.entries:
            if e.fqn not in values:
                raise KeyError(f"state dict is missing {e.fqn!r}")
            lo, hi, so = _local_piece(u, e, R)
            v = values[e.fqn]
            if full:
                if e.tp_kind == "row":
                    n = e.shape[0]
                    v = v[tpr * n:(tpr + 1) * n]
                elif e.tp_kind == "col":
                    n = e.shape[1]
                    v = v[:, tpr * n:(tpr + 1) * n]
                if tuple(v.shape) != tuple(e.shape):
                    raise ValueError(f"{e.fqn}: shape {tuple(v.shape)} != expected {tuple(e.shape)}")
                v = v.reshape(-1)[lo:hi]
            elif v.dim() != 1 or v.numel() != hi - lo:
                raise ValueError(f"{e.fqn}: shard holds {v.numel()} values, this rank owns {hi - lo}; the "
                                 "checkpoint was saved with another topology")
            shard[so:so + (hi - lo)].copy_(v.to(dev, torch.float32))
        targets[ui].copy_(shard.to(targets[ui].dtype))


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
