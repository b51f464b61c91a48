"""The training orchestrator.

Construction order (``src/training/trainer.py:90-151``): process context ->
config validation -> per-dp-rank seed -> logger -> model -> tensor
parallelism -> activation checkpointing -> sharding engine -> optimizer ->
scheduler -> datasets/loaders -> cross-rank batch-config check -> resume.

Differences: the model is always handed to the sharding engine (also at
dp = 1), so GPU runs compute in bf16 from flat buffers with an fp32 master
and the fused optimizer; the model is built on the CPU and only shards reach
the GPU, instead of a full fp32 model per rank; ``resume_from`` may name a run
directory, in which case the newest valid checkpoint in it is used (the
reference documented that but validated the given path as a checkpoint).
"""

from __future__ import annotations

import contextlib
import os
import time
from collections.abc import Iterator
from typing import Any

import torch
import torch.distributed as dist
from torch.utils.data import DataLoader, Dataset

from ..checkpointing.checkpoint import load_checkpoint, save_checkpoint
from ..checkpointing.recovery import find_latest_valid_checkpoint, require_valid_checkpoint
from ..config import TrainingConfig
from ..data.dataloader import build_dataloader
from ..data.dataset import PackedTokenDataset, SyntheticTokenDataset, UniformTokenDataset
from ..models.transformer import TransformerBlock, build_model
from ..observability.logging import build_logger
from ..observability.metrics import reset_peak_memory
from ..observability.profiler import build_profiler
from ..parallel.fsdp import apply_activation_checkpointing, wrap_model_with_fsdp
from ..parallel.process_groups import ProcessContext, build_process_context
from ..parallel.tensor_parallel import apply_tensor_parallelism
from ..utils.seed import seed_everything
from .loop import eval_step, train_step
from .optimizer import build_optimizer
from .scheduler import build_scheduler


def build_engine(config: TrainingConfig, ctx: ProcessContext) -> torch.nn.Module:
    """Model -> TP -> AC -> sharding engine, with the peer-memory transport when enabled."""
    # TP ranks must start from identical full weights: seed by the base seed here
    torch.manual_seed(config.seed)
    model = build_model(config.model)
    use_peer = (ctx.device.type == "cuda" and config.kernels.fused_comm and ctx.world_size > 1)
    tp_comm = dp_comm = None
    if use_peer:
        from ..parallel import symmetric
        tp_comm, dp_comm = symmetric.build_comms(ctx, config)
    apply_tensor_parallelism(model, ctx.tp_group if ctx.dims.tp_size > 1 else None,
                             sequence_parallel=config.parallel.sequence_parallel,
                             loss_parallel=config.parallel.loss_parallel, fused=use_peer)
    if getattr(model, "tp", None) is not None and tp_comm is not None:
        model.tp.comm = tp_comm
    if config.parallel.activation_checkpointing:
        apply_activation_checkpointing(model, {TransformerBlock})
    engine = wrap_model_with_fsdp(model, ctx, config.parallel, {TransformerBlock}, comm=dp_comm)
    if ctx.device.type == "cuda":
        model.rope_cos = model.rope_cos.to(ctx.device)
        model.rope_sin = model.rope_sin.to(ctx.device)
    return engine


class Trainer:
    def __init__(self, config: TrainingConfig, ctx: ProcessContext | None = None,
                 train_dataset: Dataset | None = None, val_dataset: Dataset | None = None,
                 gpu_type: str = "b200") -> None:
        self.config = config
        self.gpu_type = gpu_type
        self.ctx = ctx or build_process_context(config.parallel.tp_size, config.parallel.dp_size,
                                                config.backend)
        config.validate(self.ctx.world_size, self.ctx.dims.dp_size, self.ctx.dims.tp_size)
        seed_everything(config.seed, self.ctx.dims.dp_rank, deterministic=False)
        self.logger = build_logger(self.ctx.rank, config.run_id)
        self.model = build_engine(config, self.ctx)
        self.model.module.return_logits = False
        seed_everything(config.seed, self.ctx.dims.dp_rank, deterministic=False)
        self.optimizer = build_optimizer(self.model, config.optimizer)
        self.scheduler = build_scheduler(self.optimizer, config.scheduler, config.optimizer.lr)
        self.train_dataset = train_dataset or self._default_dataset("train")
        self.val_dataset = val_dataset or self._default_dataset("val")
        self.train_loader = self._loader(self.train_dataset, config.data.shuffle)
        self.val_loader = self._loader(self.val_dataset, False)
        self._train_iter: Iterator[Any] | None = None
        self._epoch = 0
        self._assert_consistent_global_batch()
        self.step = 0
        if config.resume_from:
            path = config.resume_from
            if not os.path.exists(os.path.join(path, "_SUCCESS")):
                latest = find_latest_valid_checkpoint(path, expected_config=config.to_dict())
                if latest is not None:
                    path = latest
            require_valid_checkpoint(path, expected_config=config.to_dict(), deep=False)
            self.step = load_checkpoint(self.model, self.optimizer, self.scheduler, path, self.ctx)
            self._fast_forward_data(self.step)
            self.logger.info("resumed", step=self.step, path=path)

    def _default_dataset(self, split: str) -> Dataset:
        c = self.config
        n = 4096 if split == "train" else 256
        seed = c.seed + (0 if split == "train" else 7)
        if c.data.dataset_path == "synthetic":
            return SyntheticTokenDataset(c.model.vocab_size, c.data.seq_len, n, seed)
        if c.data.dataset_path == "uniform":
            return UniformTokenDataset(c.model.vocab_size, c.data.seq_len, n, seed)
        return PackedTokenDataset(c.data.dataset_path, c.data.seq_len)

    def _loader(self, ds: Dataset, shuffle: bool) -> DataLoader:
        c = self.config
        return build_dataloader(ds, c.data.micro_batch_size, self.ctx.dims.dp_size,
                                self.ctx.dims.dp_rank, shuffle=shuffle, seed=c.seed,
                                num_workers=c.data.num_workers)

    def _assert_consistent_global_batch(self) -> None:
        c = self.config
        local = torch.tensor([c.data.micro_batch_size, c.grad_accum_steps, c.data.global_batch_size],
                             dtype=torch.long, device=self.ctx.device)
        if dist.is_initialized() and self.ctx.world_size > 1:
            mx = local.clone()
            dist.all_reduce(mx, op=dist.ReduceOp.MAX)
            if not torch.equal(mx, local):
                raise RuntimeError(
                    f"[rank {self.ctx.rank}] batch config differs across ranks: local="
                    f"{local.tolist()} max={mx.tolist()}; every rank needs the same settings.")

    def _batch_iterator(self) -> Iterator[Any]:
        while True:
            sampler = self.train_loader.sampler
            if hasattr(sampler, "set_epoch"):
                sampler.set_epoch(self._epoch)
            yield from self.train_loader
            self._epoch += 1

    def _fast_forward_data(self, step: int) -> None:
        self._epoch = 0
        self._train_iter = self._batch_iterator()
        for _ in range(step * self.config.grad_accum_steps):
            next(self._train_iter)

    def _next_window(self) -> tuple[list[Any], float]:
        if self._train_iter is None:
            self._train_iter = self._batch_iterator()
        t0 = time.perf_counter()
        window = [next(self._train_iter) for _ in range(self.config.grad_accum_steps)]
        return window, time.perf_counter() - t0

    def _eval_windows(self) -> list[Any]:
        out = []
        for i, b in enumerate(self.val_loader):
            if i >= self.config.eval_steps:
                break
            out.append(b)
        return out

    def train(self) -> None:
        c = self.config
        self.logger.info("train_start", start_step=self.step, max_steps=c.max_steps,
                         tp_size=self.ctx.dims.tp_size, dp_size=self.ctx.dims.dp_size,
                         world_size=self.ctx.world_size)
        reset_peak_memory(self.ctx.device)
        prof = None
        pctx: contextlib.AbstractContextManager = contextlib.nullcontext()
        if c.profile_steps > 0 and self.ctx.is_rank0:
            prof = build_profiler(f"traces/{c.run_id}", c.warmup_profile_steps, c.profile_steps)
            pctx = prof
        try:
            with pctx:
                while self.step < c.max_steps:
                    window, wait = self._next_window()
                    m = train_step(self.model, window, self.optimizer, self.scheduler, self.ctx, c,
                                   gpu_type=self.gpu_type, data_wait_s=wait)
                    self.step += 1
                    if prof is not None:
                        prof.step()
                    if self.step % c.log_interval == 0:
                        self.logger.metric("step", step=self.step, **_metric_fields(m))
                        reset_peak_memory(self.ctx.device)
                    if c.eval_interval > 0 and self.step % c.eval_interval == 0:
                        val = eval_step(self.model, self._eval_windows(), self.ctx, c)
                        self.logger.metric("eval", step=self.step, val_loss=val)
                    if c.save_interval > 0 and self.step % c.save_interval == 0:
                        path = save_checkpoint(self.model, self.optimizer, self.scheduler, self.step,
                                               c, self.ctx)
                        self.logger.info("checkpoint", step=self.step, path=path)
        except KeyboardInterrupt:
            self.logger.warning("interrupted", step=self.step)
            save_checkpoint(self.model, self.optimizer, self.scheduler, self.step, c, self.ctx)
            self.logger.info("checkpoint_on_interrupt", step=self.step)
            raise
        self.logger.info("train_done", step=self.step)


def _metric_fields(m: Any) -> dict[str, Any]:
    return {"loss": round(m.loss, 5), "ppl": round(m.perplexity(), 3),
            "grad_norm": round(m.grad_norm, 4), "lr": m.learning_rate,
            "tok_per_s": round(m.tokens_per_second, 1),
            "mfu": round(m.mfu, 4) if m.mfu is not None else None,
            "step_time_s": round(m.step_time_s, 4),
            "device_time_s": round(m.device_time_s, 4) if m.device_time_s is not None else None,
            "data_wait_s": round(m.data_wait_s, 4),
            "peak_mem_mb": round(m.peak_memory_bytes / 1e6, 1)}
