"""Gradient norm, clipping and the collective finite check.

Semantics of ``src/training/grad_utils.py:47-230``:

* global L2 norm over every parameter of the (sharded, TP-split) model, with
  TP-replicated parameters counted once; ``coef = max_norm / (norm + 1e-6)``
  applied when below 1; ``max_norm <= 0`` disables clipping;
* ``grad_finite_check`` raises ``GradNotFiniteError`` on every rank together
  when any rank holds a non-finite gradient (MIN all-reduce over the world).

For the sharded engine the norm is one fp32 scalar all-reduce over the world
of per-rank partial sums of squares; ``device_clip_state`` turns it into the
device-resident ``[coef, finite]`` pair the fused optimizer consumes, so the
step needs no host round trip until the metrics are read.
"""

from __future__ import annotations

from collections.abc import Iterable
from typing import Union

import torch
import torch.distributed as dist
import torch.nn as nn

from ..parallel.fsdp import FullyShardedModel
from ..parallel.tensor_parallel import tp_param_kind

ParamsOrModule = Union[nn.Module, Iterable[torch.nn.Parameter]]  # noqa: UP007


class GradNotFiniteError(RuntimeError):
    """A gradient held NaN/Inf on at least one rank; the update was not applied."""


def _grad_of(p: torch.Tensor) -> torch.Tensor | None:
    return p.grad


def sharded_total_norm(model: FullyShardedModel) -> torch.Tensor:
    """Device scalar: global L2 norm of the model's gradients (all ranks agree)."""
    sq = model.grad_norm_sq_local().reshape(1).clone()
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(sq)
    return sq.sqrt()[0]


def device_clip_state(total_norm: torch.Tensor, max_norm: float) -> torch.Tensor:
    """``[coef, finite]`` on the norm's device: ``coef = min(1, max/(norm+1e-6))``."""
    finite = torch.isfinite(total_norm)
    if max_norm > 0:
        coef = torch.clamp(max_norm / (total_norm + 1e-6), max=1.0)
    else:
        coef = torch.ones_like(total_norm)
    coef = torch.where(finite, coef, torch.zeros_like(coef))
    return torch.stack([coef, finite.float()]).float()


def clip_grad_norm_(target: ParamsOrModule, max_norm: float, norm_type: float = 2.0,
                    tp_group: dist.ProcessGroup | None = None) -> float:
    """Clip in place and return the pre-clip global norm."""
    if isinstance(target, FullyShardedModel):
        if norm_type != 2.0:
            raise ValueError("the sharded engine clips by the L2 norm only")
        norm = sharded_total_norm(target)
        state = device_clip_state(norm, max_norm)
        for u in target.units:
            u.grad_shard.mul_(state[0] if bool(state[1]) else 1.0)
        return float(norm)
    params = list(target.parameters()) if isinstance(target, nn.Module) else list(target)
    model = target if isinstance(target, nn.Module) else None
    tp = getattr(model, "tp", None) if model is not None else None
    if tp is not None and tp.size > 1:
        return _tp_aware_clip(model, max_norm, norm_type, tp_group or tp.group)
    grads = [p.grad for p in params if p.grad is not None]
    if not grads:
        return 0.0
    if max_norm <= 0:
        return float(torch.norm(torch.stack([torch.norm(g.detach(), norm_type) for g in grads]),
                                norm_type))
    return float(torch.nn.utils.clip_grad_norm_(params, max_norm, norm_type))


def _tp_aware_clip(model: nn.Module, max_norm: float, norm_type: float,
                   tp_group: dist.ProcessGroup | None) -> float:
    if norm_type != 2.0:
        raise ValueError(f"TP-aware clipping supports L2 only, got norm_type={norm_type}.")
    tp_size = dist.get_world_size(tp_group) if tp_group is not None else 1
    sq = torch.zeros((), dtype=torch.float32)
    seen: set[int] = set()
    params = []
    for fqn, p in model.named_parameters():
        if p.grad is None or id(p) in seen:
            continue
        seen.add(id(p))
        params.append(p)
        part = p.grad.detach().float().pow(2).sum().cpu()
        sq = sq + (part if tp_param_kind(fqn, model) != "rep" else part / tp_size)
    if tp_size > 1:
        dist.all_reduce(sq, group=tp_group)
    total = float(sq.sqrt())
    if max_norm > 0:
        coef = max_norm / (total + 1e-6)
        if coef < 1.0:
            for p in params:
                p.grad.mul_(coef)
    return total


def grad_finite_check(target: ParamsOrModule, group: dist.ProcessGroup | None = None,
                      device: torch.device | None = None) -> bool:
    """Raise :class:`GradNotFiniteError` on all ranks if any rank has a bad gradient."""
    ok = 1
    if isinstance(target, FullyShardedModel):
        ok = int(bool(torch.isfinite(target.grad_norm_sq_local())))
        device = device or target.device
    else:
        params = list(target.parameters()) if isinstance(target, nn.Module) else list(target)
        for p in params:
            if p.grad is not None and not torch.isfinite(p.grad).all():
                ok = 0
                break
    flag = torch.tensor([ok], dtype=torch.int32, device=device)
    if dist.is_initialized():
        dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
    if int(flag.item()) == 0:
        rank = dist.get_rank() if dist.is_initialized() else 0
        raise GradNotFiniteError(
            f"[rank {rank}] non-finite gradient on at least one rank (local ok={ok}); the "
            "optimizer step was not applied. Usual causes: learning rate too high, no clipping, "
            "fp16 overflow (use bf16), a bad batch.")
    return True
