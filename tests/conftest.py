"""Shared fixtures; the ``gpu`` marker selects tests that need a B200."""

from __future__ import annotations

import os
import sys

import pytest
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (sm_100a) and the native extension")
    config.addinivalue_line("markers", "slow: long-running CPU test")


@pytest.fixture()
def single_process_pg():
    """A world-size-1 gloo group, torn down after the test."""
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29555")
    os.environ.setdefault("RANK", "0")
    os.environ.setdefault("WORLD_SIZE", "1")
    if not dist.is_initialized():
        dist.init_process_group(backend="gloo", world_size=1, rank=0)
    yield
    if dist.is_initialized():
        dist.destroy_process_group()
