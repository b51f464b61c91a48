"""NVTX ranges for step phases and transformer blocks (for nsys / ncu range filters).

Off unless ``DTB_NVTX=1``: each range is a host call per block and phase, so
it is kept out of timed runs by default.  Ranges: ``forward``, ``backward``,
``optimizer`` per step (``train_step``) and ``block{i}.fwd`` / ``block{i}.bwd``
per transformer block (the sharding engine's hooks).
"""
from __future__ import annotations

import contextlib
import os

import torch

_ENABLED = os.environ.get("DTB_NVTX", "0") == "1"


def enabled() -> bool:
    return _ENABLED and torch.cuda.is_available()


def push(name: str) -> None:
    if enabled():
        torch.cuda.nvtx.range_push(name)


def pop() -> None:
    if enabled():
        torch.cuda.nvtx.range_pop()


@contextlib.contextmanager
def nvtx_range(name: str):
    push(name)
    try:
        yield
    finally:
        pop()
