"""Optimizers: sharded fused AdamW over the engine's flat fp32 shards, LAMB.

``ShardedAdamW`` updates each unit's fp32 master shard from its fp32 gradient
shard and writes the ``param_dtype`` shard the next all-gather reads.  On CUDA
that is one ``adamw`` kernel per (unit, decay segment); it reads the clip
coefficient and the finite flag from device memory, so clipping and the
skip-on-NaN rule need no host synchronisation (the reference used torch's
fused AdamW after a host-side finite check, ``src/training/optimizer.py:163-189``
and ``src/training/loop.py:166-168``).

Weight decay applies to matrices (>= 2-D) only.  The reference meant that too
(``build_param_groups``, ``:38-73``) but, because it grouped parameters after
FSDP had flattened them to 1-D, it applied no decay at all under FSDP;
``OptimizerConfig.decay_flat_params_under_fsdp = True`` reproduces that.

``LAMB`` keeps the reference's update (``:76-160``) for plain modules; on the
sharded engine the trust ratio uses the exact per-parameter norms (shard
partial sums all-reduced over the shard group).
"""

from __future__ import annotations

from typing import Any

import torch
import torch.distributed as dist
import torch.nn as nn
from torch.optim import Optimizer

from ..parallel.fsdp import FullyShardedModel


def build_param_groups(model: nn.Module, weight_decay: float) -> list[dict[str, Any]]:
    decay, no_decay, seen = [], [], set()
    for p in model.parameters():
        if not p.requires_grad or id(p) in seen:
            continue
        seen.add(id(p))
        (decay if p.dim() >= 2 else no_decay).append(p)
    groups = []
    if decay:
        groups.append({"params": decay, "weight_decay": weight_decay})
    if no_decay:
        groups.append({"params": no_decay, "weight_decay": 0.0})
    return groups


class LAMB(Optimizer):
    """Layer-wise adaptive moments: Adam direction scaled by ``||w|| / ||update||``."""

    def __init__(self, params: Any, lr: float = 1e-3, betas: tuple[float, float] = (0.9, 0.999),
                 eps: float = 1e-6, weight_decay: float = 0.0) -> None:
        if lr <= 0:
            raise ValueError(f"LAMB: lr must be > 0, got {lr}.")
        super().__init__(params, {"lr": lr, "betas": betas, "eps": eps, "weight_decay": weight_decay})

    @torch.no_grad()
    def step(self, closure: Any = None) -> Any:  # type: ignore[override]
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            b1, b2 = group["betas"]
            for p in group["params"]:
                if p.grad is None:
                    continue
                st = self.state[p]
                if not st:
                    st["step"] = 0
                    st["exp_avg"] = torch.zeros_like(p)
                    st["exp_avg_sq"] = torch.zeros_like(p)
                st["step"] += 1
                upd = _lamb_direction(p, p.grad, st, b1, b2, group["eps"], group["weight_decay"])
                w_norm, u_norm = p.norm(2), upd.norm(2)
                trust = torch.where((w_norm > 0) & (u_norm > 0), w_norm / u_norm, torch.ones_like(w_norm))
                p.add_(upd * trust, alpha=-group["lr"])
        return loss


def _lamb_direction(p, g, st, b1, b2, eps, wd):
    m, v, t = st["exp_avg"], st["exp_avg_sq"], st["step"]
    m.mul_(b1).add_(g, alpha=1 - b1)
    v.mul_(b2).addcmul_(g, g, value=1 - b2)
    upd = (m / (1 - b1 ** t)) / ((v / (1 - b2 ** t)).sqrt() + eps)
    return upd.add(p, alpha=wd) if wd != 0 else upd


class ShardedAdamW(Optimizer):
    """AdamW (decoupled decay, torch semantics) on the engine's flat shards."""

    def __init__(self, model: FullyShardedModel, lr: float, betas: tuple[float, float],
                 eps: float, weight_decay: float, decay_flat: bool = False, name: str = "adamw") -> None:
        self.model = model
        self.decay_flat = decay_flat
        self.kind = name
        params = [u.master for u in model.units]
        super().__init__(params, {"lr": lr, "betas": tuple(betas), "eps": eps,
                                  "weight_decay": weight_decay})
        # device-side [clip_coef, finite] consumed by the update kernel
        self._clip_state: torch.Tensor | None = None

    def zero_grad(self, set_to_none: bool = True) -> None:  # noqa: ARG002
        self.model.zero_grad_buffers()

    def set_clip_state(self, state: torch.Tensor | None) -> None:
        self._clip_state = state

    def _segments(self, u) -> list[tuple[int, int, bool]]:
        lo, hi = u.shard_range(self.model.shard_rank)
        cut = min(max(u.decay_end, lo), hi)
        segs = []
        if cut > lo:
            segs.append((0, cut - lo, not self.decay_flat))
        if hi > cut:
            segs.append((cut - lo, hi - lo, False))
        return segs

    @torch.no_grad()
    def step(self, closure: Any = None) -> Any:  # type: ignore[override]
        loss = closure() if closure is not None else None
        group = self.param_groups[0]
        lr, (b1, b2), eps, wd = group["lr"], group["betas"], group["eps"], group["weight_decay"]
        clip = self._clip_state
        for u in self.model.units:
            st = self.state[u.master]
            if not st:
                st["step"] = torch.zeros((), dtype=torch.float32)
                st["exp_avg"] = torch.zeros_like(u.master)
                st["exp_avg_sq"] = torch.zeros_like(u.master)
            st["step"] += 1
            t = int(st["step"].item())
            if self.kind == "lamb":
                self._lamb_unit(u, st, lr, b1, b2, eps, wd, t, clip)
                continue
            for a, b, dec in self._segments(u):
                m, v = st["exp_avg"][a:b], st["exp_avg_sq"][a:b]
                p, g, out = u.master[a:b], u.grad_shard[a:b], u.param_shard[a:b]
                w = wd if dec else 0.0
                if p.is_cuda:
                    from ..ops._ext import native
                    native().adamw(p, g, m, v, out, clip, lr, b1, b2, eps, w, t)
                else:
                    _adamw_ref(p, g, m, v, out, clip, lr, b1, b2, eps, w, t)
        self.model.after_optimizer_step()
        return loss

    def _lamb_unit(self, u, st, lr, b1, b2, eps, wd, t, clip) -> None:
        lo, hi = u.shard_range(self.model.shard_rank)
        g = u.grad_shard * (clip[0] if clip is not None else 1.0)
        if clip is not None and clip[1] == 0:
            return
        p = u.master
        m, v = st["exp_avg"], st["exp_avg_sq"]
        m.mul_(b1).add_(g, alpha=1 - b1)
        v.mul_(b2).addcmul_(g, g, value=1 - b2)
        upd = (m / (1 - b1 ** t)) / ((v / (1 - b2 ** t)).sqrt() + eps)
        norms = torch.zeros(len(u.entries), 2, dtype=torch.float32, device=p.device)
        segs = []
        for i, e in enumerate(u.entries):
            a, b = max(lo, e.offset), min(hi, e.offset + e.numel)
            if b <= a:
                segs.append(None)
                continue
            s = slice(a - lo, b - lo)
            if e.decay and not self.decay_flat and wd != 0:
                upd[s].add_(p[s], alpha=wd)
            norms[i, 0] = p[s].float().pow(2).sum()
            norms[i, 1] = upd[s].float().pow(2).sum()
            segs.append(s)
        if self.model.shard_world > 1:
            dist.all_reduce(norms, group=self.model.comm.group)
        for i, s in enumerate(segs):
            if s is None:
                continue
            wn, un = norms[i, 0].sqrt(), norms[i, 1].sqrt()
            trust = torch.where((wn > 0) & (un > 0), wn / un, torch.ones_like(wn))
            p[s].add_(upd[s] * trust, alpha=-lr)
        u.param_shard.copy_(p.to(u.param_shard.dtype))


def _adamw_ref(p, g, m, v, out, clip, lr, b1, b2, eps, wd, t) -> None:
    if clip is not None:
        if float(clip[1]) == 0.0:
            return
        g = g * clip[0]
    p.mul_(1 - lr * wd)
    m.mul_(b1).add_(g, alpha=1 - b1)
    v.mul_(b2).addcmul_(g, g, value=1 - b2)
    denom = (v.sqrt() / (1 - b2 ** t) ** 0.5).add_(eps)
    p.addcdiv_(m, denom, value=-lr / (1 - b1 ** t))
    out.copy_(p.to(out.dtype))


def build_optimizer(model: nn.Module, cfg) -> Optimizer:
    name = cfg.name.lower()
    if name not in ("adamw", "lamb"):
        raise ValueError(f"Unknown optimizer name={cfg.name!r}; valid: 'adamw', 'lamb'.")
    if isinstance(model, FullyShardedModel):
        return ShardedAdamW(model, cfg.lr, cfg.betas, cfg.eps, cfg.weight_decay,
                            decay_flat=getattr(cfg, "decay_flat_params_under_fsdp", False), name=name)
    groups = build_param_groups(model, cfg.weight_decay)
    if name == "adamw":
        fused = bool(cfg.fused and torch.cuda.is_available()
                     and all(p.is_cuda for g in groups for p in g["params"]))
        return torch.optim.AdamW(groups, lr=cfg.lr, betas=cfg.betas, eps=cfg.eps, fused=fused)
    return LAMB(groups, lr=cfg.lr, betas=cfg.betas, eps=cfg.eps)
