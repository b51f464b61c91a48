"""Process-group bootstrap and the explicit ``ProcessContext``.

Every rank is one OS process bound to one GPU.  ``torch.distributed`` (NCCL on
GPU, gloo on CPU) is only the bootstrap and scalar transport; the hot
collectives run as this package's own peer-memory kernels
(:mod:`.symmetric`).  API and behaviour follow
``src/parallelism/process_groups.py:51-183``; the default collective timeout
is shorter (300 s instead of 1800 s) so ranks waiting on a dead peer end with
an error in minutes, and it can be set per call.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from datetime import timedelta

import torch
import torch.distributed as dist
from torch.distributed.device_mesh import DeviceMesh

from ..utils.env import LaunchEnv, read_launch_env, select_device
from .mesh import (ParallelDims, build_device_mesh, format_mesh_layout, get_dp_group,
                   get_parallel_dims, get_tp_group)

DEFAULT_TIMEOUT_S = int(os.environ.get("DTB_PG_TIMEOUT_S", "300"))


@dataclass(frozen=True)
class ProcessContext:
    env: LaunchEnv
    device: torch.device
    mesh: DeviceMesh
    dims: ParallelDims
    dp_group: dist.ProcessGroup
    tp_group: dist.ProcessGroup

    @property
    def rank(self) -> int:
        return self.dims.global_rank

    @property
    def world_size(self) -> int:
        return self.dims.world_size

    @property
    def is_rank0(self) -> bool:
        return self.dims.global_rank == 0

    @property
    def is_dp_rank0(self) -> bool:
        return self.dims.dp_rank == 0

    def barrier(self) -> None:
        if dist.is_initialized():
            if self.device.type == "cuda":
                dist.barrier(device_ids=[self.device.index])
            else:
                dist.barrier()


def init_distributed(backend: str = "nccl", timeout_seconds: int = DEFAULT_TIMEOUT_S) -> LaunchEnv:
    """Initialise the default process group once (idempotent)."""
    env = read_launch_env(backend=backend)
    if not dist.is_initialized() and env.world_size == 1:
        # a plain `python train.py` run: rendezvous with ourselves on a free local port
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        if "MASTER_PORT" not in os.environ:
            import socket
            with socket.socket() as s:
                s.bind(("127.0.0.1", 0))
                os.environ["MASTER_PORT"] = str(s.getsockname()[1])
    if not dist.is_initialized():
        kwargs = {}
        if backend == "nccl":
            # Bind the communicator to this rank's GPU up front (eager init).
            torch.cuda.set_device(env.local_rank)
            kwargs["device_id"] = torch.device("cuda", env.local_rank)
        dist.init_process_group(backend=backend, world_size=env.world_size, rank=env.rank,
                                timeout=timedelta(seconds=timeout_seconds), **kwargs)
    return env


def build_process_context(tp_size: int, dp_size: int = -1, backend: str = "nccl",
                          timeout_seconds: int = DEFAULT_TIMEOUT_S,
                          verbose: bool = True) -> ProcessContext:
    env = init_distributed(backend=backend, timeout_seconds=timeout_seconds)
    device = select_device(env)
    mesh = build_device_mesh(tp_size, dp_size, "cuda" if device.type == "cuda" else "cpu")
    ctx = ProcessContext(env, device, mesh, get_parallel_dims(mesh), get_dp_group(mesh),
                         get_tp_group(mesh))
    if ctx.is_rank0 and verbose:
        print(format_mesh_layout(mesh), flush=True)
    return ctx


def destroy_distributed() -> None:
    from . import symmetric  # release peer mappings before the process group goes
    symmetric.release_all()
    if dist.is_initialized():
        dist.destroy_process_group()
