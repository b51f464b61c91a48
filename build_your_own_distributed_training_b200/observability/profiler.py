"""torch.profiler window, trace export and the communication share of CUDA time.

``build_profiler`` / ``communication_fraction`` / ``text_summary`` /
``export_chrome_trace`` behave as ``src/observability/profiler.py:35-141``.
The collective-name hints also match this package's own peer-memory kernels
(``peer_`` prefix), and ``fused_kernel_share`` reports fused
GEMM+collective kernels separately, since their time cannot be split into
"compute" and "communication" by name.
"""

from __future__ import annotations

import os
from dataclasses import dataclass

import torch
from torch.profiler import ProfilerActivity, profile, schedule, tensorboard_trace_handler

COMM_HINTS = ("nccl", "all_reduce", "allreduce", "all_gather", "allgather", "reduce_scatter",
              "reducescatter", "broadcast", "c10d", "peer_", "dev_barrier")
FUSED_HINTS = ("gemm_ar", "gemm_rs", "ag_gemm")


@dataclass
class CommComputeBreakdown:
    total_cuda_us: float
    comm_cuda_us: float
    compute_cuda_us: float
    comm_fraction: float
    fused_cuda_us: float = 0.0


def build_profiler(output_dir: str, warmup_steps: int, profile_steps: int, *,
                   record_memory: bool = True) -> profile:
    os.makedirs(output_dir, exist_ok=True)
    acts = [ProfilerActivity.CPU]
    if torch.cuda.is_available():
        acts.append(ProfilerActivity.CUDA)
    return profile(activities=acts,
                   schedule=schedule(wait=max(0, warmup_steps - 1), warmup=1, active=profile_steps,
                                     repeat=1),
                   on_trace_ready=tensorboard_trace_handler(output_dir), record_shapes=True,
                   profile_memory=record_memory, with_stack=False)


def export_chrome_trace(prof: profile, path: str) -> None:
    os.makedirs(os.path.dirname(path) or ".", exist_ok=True)
    prof.export_chrome_trace(path)


def text_summary(prof: profile, row_limit: int = 20) -> str:
    key = "self_cuda_time_total" if torch.cuda.is_available() else "self_cpu_time_total"
    return prof.key_averages().table(sort_by=key, row_limit=row_limit)


def communication_fraction(prof: profile) -> CommComputeBreakdown:
    total = comm = fused = 0.0
    for evt in prof.key_averages():
        us = float(getattr(evt, "self_device_time_total", getattr(evt, "self_cuda_time_total", 0.0)))
        total += us
        name = evt.key.lower()
        if any(h in name for h in FUSED_HINTS):
            fused += us
        elif any(h in name for h in COMM_HINTS):
            comm += us
    return CommComputeBreakdown(total, comm, total - comm - fused,
                                comm / total if total > 0 else 0.0, fused)
