"""Run a function on N gloo ranks in spawned processes (CUDA hidden).

A child's exception propagates to pytest, so a failing rank fails the test
instead of hanging it; the process group has a short timeout so a rank that
dies leaves the others with an error, not a hang.
"""

from __future__ import annotations

import os
import socket
from collections.abc import Callable
from datetime import timedelta
from typing import Any

import torch.distributed as dist
import torch.multiprocessing as mp


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _entry(rank: int, world: int, port: int, fn: Callable[..., None], args: tuple) -> None:
    os.environ.update({"RANK": str(rank), "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank),
                       "LOCAL_WORLD_SIZE": str(world), "MASTER_ADDR": "127.0.0.1",
                       "MASTER_PORT": str(port), "CUDA_VISIBLE_DEVICES": ""})
    import torch
    torch.set_num_threads(1)  # N ranks share the CPU cores; avoid oversubscription
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        fn(rank, world, *args)
        dist.barrier()
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def run_distributed(fn: Callable[..., None], world_size: int, *args: Any, port: int | None = None) -> None:
    os.environ["CUDA_VISIBLE_DEVICES"] = ""
    mp.spawn(_entry, args=(world_size, port or free_port(), fn, args), nprocs=world_size, join=True)
