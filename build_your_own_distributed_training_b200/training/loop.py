"""One optimizer step (``train_step``) and evaluation (``eval_step``).

Order of operations (``src/training/loop.py:94-235``): zero grads; for each
micro-batch move it to the device, run forward under ``no_sync`` unless it is
the last one, backward ``loss / accum``; finite check over the world; clip;
optimizer step; scheduler step; metrics with ``global_tokens = local * dp``.

Differences on the sharded engine (GPU path): the model already computes in
``param_dtype`` (no autocast); the norm, the clip coefficient and the finite
flag stay on the device and the fused optimizer consumes them, so the one
host synchronisation per step is the read of ``[loss, norm, finite]`` the
metrics need.  A non-finite gradient still raises
:class:`~.grad_utils.GradNotFiniteError` on every rank before the scheduler
steps, and the device skipped the parameter update.  Step time is reported
twice: host wall clock (the reference's number) and CUDA-event device time,
max over ranks.
"""

from __future__ import annotations

import contextlib
import time
from collections.abc import Mapping, Sequence
from typing import Any

import torch
import torch.distributed as dist
import torch.nn as nn

from ..observability.nvtx import nvtx_range
from ..observability.metrics import (StepMetrics, aggregate_loss, compute_mfu, compute_throughput,
                                     estimate_flops_per_token, peak_memory_bytes)
from ..parallel.fsdp import FullyShardedModel
from ..utils.dtype import autocast_dtype
from .grad_utils import (GradNotFiniteError, clip_grad_norm_, device_clip_state, grad_finite_check,
                         sharded_total_norm)

Batch = Mapping[str, torch.Tensor]


def _maybe_no_sync(model: nn.Module, enabled: bool) -> contextlib.AbstractContextManager:
    if enabled and hasattr(model, "no_sync"):
        return model.no_sync()
    return contextlib.nullcontext()


def _move_batch(batch: Batch, device: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
    return (batch["input_ids"].to(device, non_blocking=True),
            batch["labels"].to(device, non_blocking=True))


def _autocast(model: nn.Module, device: torch.device, config) -> contextlib.AbstractContextManager:
    if isinstance(model, FullyShardedModel) or device.type != "cuda":
        return contextlib.nullcontext()
    return torch.autocast(device_type="cuda", dtype=autocast_dtype(config.parallel))


def train_step(model: nn.Module, micro_batches: Sequence[Batch], optimizer: torch.optim.Optimizer,
               scheduler: Any, ctx: Any, config: Any, *, gpu_type: str = "a100",
               data_wait_s: float = 0.0) -> StepMetrics:
    device = ctx.device
    accum = len(micro_batches)
    if accum == 0:
        raise ValueError("train_step received an empty micro_batch window.")
    model.train()
    optimizer.zero_grad(set_to_none=True)
    t0 = time.perf_counter()
    cuda = device.type == "cuda"
    if cuda:
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
    summed = torch.zeros((), device=device)
    local_tokens = 0
    for i, batch in enumerate(micro_batches):
        ids, labels = _move_batch(batch, device)
        local_tokens += ids.numel()
        with _maybe_no_sync(model, enabled=i < accum - 1):
            with _autocast(model, device, config), nvtx_range("forward"):
                _, loss = model(ids, labels=labels)
            assert loss is not None, "the model must return a loss when labels are given"
            scaled = loss / accum
            with nvtx_range("backward"):
                scaled.backward()
        summed = summed + scaled.detach().float()

    sharded = isinstance(model, FullyShardedModel)
    if sharded:
        with nvtx_range("optimizer"):
            norm = sharded_total_norm(model)
            state = device_clip_state(norm, config.max_grad_norm)
            optimizer.set_clip_state(state)  # type: ignore[attr-defined]
            optimizer.step()
        loss_t = summed.reshape(1).clone()
        if dist.is_initialized() and ctx.dims.dp_size > 1:
            dist.all_reduce(loss_t, group=ctx.dp_group)
            loss_t /= ctx.dims.dp_size
        host = torch.stack([loss_t[0], norm, state[1]]).cpu()  # the one host sync
        if device.type == "cuda":
            from ..parallel.symmetric import check_device_errors
            check_device_errors()  # bounded peer waits that ran out raise here
        loss_value, grad_norm, finite = float(host[0]), float(host[1]), bool(host[2] > 0)
        if not finite:
            raise GradNotFiniteError(
                f"[rank {ctx.rank}] non-finite gradient norm ({grad_norm}) on at least one rank; "
                "the update was skipped on the device. Usual causes: learning rate too high, "
                "fp16 overflow (use bf16), a bad batch.")
        scheduler.step()
    else:
        grad_finite_check(model, group=None, device=device)
        grad_norm = clip_grad_norm_(model, config.max_grad_norm, tp_group=ctx.tp_group)
        optimizer.step()
        scheduler.step()
        loss_value = aggregate_loss(summed, ctx.dp_group)
    device_time = None
    if cuda:
        ev1.record()
        ev1.synchronize()
        dt = torch.tensor([ev0.elapsed_time(ev1) / 1e3], device=device)
        if dist.is_initialized() and dist.get_world_size() > 1:
            dist.all_reduce(dt, op=dist.ReduceOp.MAX)
        device_time = float(dt.item())
    step_time = time.perf_counter() - t0
    global_tokens = local_tokens * ctx.dims.dp_size
    tps = compute_throughput(global_tokens, step_time)
    mfu = compute_mfu(tps, estimate_flops_per_token(config.model), ctx.world_size, gpu_type)
    return StepMetrics(loss=loss_value, grad_norm=grad_norm,
                       learning_rate=float(scheduler.get_last_lr()[0]), tokens_per_second=tps,
                       step_time_s=step_time, data_wait_s=data_wait_s, mfu=mfu,
                       peak_memory_bytes=peak_memory_bytes(device), device_time_s=device_time)


@torch.no_grad()
def eval_step(model: nn.Module, micro_batches: Sequence[Batch], ctx: Any, config: Any) -> float:
    """Mean loss over the window, averaged over dp."""
    if len(micro_batches) == 0:
        return 0.0
    model.eval()
    total = torch.zeros((), device=ctx.device)
    for batch in micro_batches:
        ids, labels = _move_batch(batch, ctx.device)
        with _autocast(model, ctx.device, config):
            _, loss = model(ids, labels=labels)
        total = total + loss.detach().float()
    return aggregate_loss(total / len(micro_batches), ctx.dp_group)
