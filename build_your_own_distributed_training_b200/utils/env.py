"""Launch-environment parsing and device binding.

Reads the torchrun variables with single-process defaults and checks, before
any collective exists, that an NCCL launch has a GPU for its local rank
(reference ``src/utils/env.py:29-117``).  One process drives one GPU.
"""

from __future__ import annotations

import os
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class LaunchEnv:
    rank: int
    world_size: int
    local_rank: int
    local_world_size: int
    master_addr: str
    master_port: str
    backend: str


def read_launch_env(backend: str = "nccl") -> LaunchEnv:
    """Parse ``RANK``/``WORLD_SIZE``/``LOCAL_RANK``/... from the environment.

    Raises ``RuntimeError`` when ``backend == "nccl"`` and either CUDA is not
    available or ``LOCAL_RANK`` has no device, so a bad launch fails at once
    with the reason instead of hanging in the first collective.
    """
    env = os.environ
    rank = int(env.get("RANK", "0"))
    world = int(env.get("WORLD_SIZE", "1"))
    local_rank = int(env.get("LOCAL_RANK", "0"))
    local_world = int(env.get("LOCAL_WORLD_SIZE", str(world)))
    if backend == "nccl":
        if not torch.cuda.is_available():
            raise RuntimeError(
                f"[rank {rank}] backend='nccl' needs CUDA but torch.cuda.is_available() is "
                "False; use backend='gloo' on CPU."
            )
        n = torch.cuda.device_count()
        if local_rank >= n:
            raise RuntimeError(
                f"[rank {rank}] LOCAL_RANK={local_rank} but only {n} CUDA devices are "
                "visible; every local rank needs its own GPU (check nproc_per_node and "
                "CUDA_VISIBLE_DEVICES)."
            )
    return LaunchEnv(rank, world, local_rank, local_world,
                     env.get("MASTER_ADDR", "127.0.0.1"), env.get("MASTER_PORT", "29500"),
                     backend)


def select_device(env: LaunchEnv) -> torch.device:
    """Bind this process to ``cuda:LOCAL_RANK`` for NCCL, else use the CPU."""
    if env.backend == "nccl" and torch.cuda.is_available():
        dev = torch.device("cuda", env.local_rank)
        torch.cuda.set_device(dev)
        return dev
    return torch.device("cpu")


def describe_versions() -> dict[str, str]:
    """Versions of torch / CUDA / NCCL / the GPU, for run logs."""
    out = {"torch": torch.__version__, "cuda": torch.version.cuda or "cpu"}
    if torch.cuda.is_available():
        out["nccl"] = ".".join(str(v) for v in torch.cuda.nccl.version())
        out["gpu"] = torch.cuda.get_device_name(0)
    return out
