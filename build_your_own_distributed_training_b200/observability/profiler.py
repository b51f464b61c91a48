"""torch.profiler window, trace export and the communication share of CUDA time.

``build_profiler`` / ``communication_fraction`` / ``text_summary`` /
``export_chrome_trace`` behave as ``src/observability/profiler.py:35-141``.
The collective-name hints also match this package's own peer-memory kernels
(``peer_`` prefix), and ``CommComputeBreakdown.fused_cuda_us`` reports fused
GEMM+collective kernels separately (``is_fused_comm_kernel``), since their time
cannot be split into "compute" and "communication" by name.
"""

from __future__ import annotations

import os
import re
from dataclasses import dataclass

import torch
from torch.profiler import ProfilerActivity, profile, schedule, tensorboard_trace_handler

COMM_HINTS = ("nccl", "all_reduce", "allreduce", "all_gather", "allgather", "reduce_scatter",
              "reducescatter", "broadcast", "c10d", "peer_", "dev_barrier")
# Kernels that do a GEMM and a collective in one launch.  The tcgen05 GEMM is one
# template, ``gemm_tcgen05_kernel<BN, STAGES, A_MN, B_MN, EPI, PAIR>``; its peer
# epilogue (EPI == 6, csrc/gemm.cu ``EPI_PEER_AR``) sums the TP group's tiles
# over NVLink (all-reduce, or reduce-scatter under sequence parallelism).
FUSED_HINTS = ("ag_gemm", "gemm_ar", "gemm_rs")
PEER_EPILOGUE_ID = 6
# template arguments as profilers print them: integers, bools as 0/1 or false/true
_ARG = r"\s*(\w+)\s*"
_GEMM_TEMPLATE = re.compile(r"gemm_tcgen05_kernel<" + ",".join([_ARG] * 5))


def is_fused_comm_kernel(name: str) -> bool:
    """True for a kernel that fuses a collective into its GEMM (by template epilogue id or name)."""
    m = _GEMM_TEMPLATE.search(name)
    if m is not None:
        return m.group(5) == str(PEER_EPILOGUE_ID)
    low = name.lower()
    return any(h in low for h in FUSED_HINTS)


def is_comm_kernel(name: str) -> bool:
    """True for a pure communication kernel (NCCL, c10d, this package's peer copies)."""
    low = name.lower()
    return not is_fused_comm_kernel(name) and any(h in low for h in COMM_HINTS)


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
        if is_fused_comm_kernel(evt.key):
            fused += us
        elif is_comm_kernel(evt.key):
            comm += us
    return CommComputeBreakdown(total, comm, total - comm - fused,
                                comm / total if total > 0 else 0.0, fused)
