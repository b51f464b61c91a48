"""Seeding and RNG-state capture.

``seed_everything`` seeds python/numpy/torch/CUDA with ``base + dp_rank`` so
data-parallel replicas differ and tensor-parallel peers agree (reference
``src/utils/seed.py:45-80``).  ``get_rng_state`` returns only tensors, ints and
tuples so a checkpoint of it loads under ``torch.load(weights_only=True)``;
the reference stored numpy's state object and its own resume failed on
torch >= 2.6 (``src/checkpointing/checkpoint.py:201-222``).
"""

from __future__ import annotations

import os
import random

import numpy as np
import torch


def seed_everything(base_seed: int, dp_rank: int = 0, deterministic: bool = False) -> int:
    seed = base_seed + dp_rank
    random.seed(seed)
    np.random.seed(seed % (2**32 - 1))
    torch.manual_seed(seed)
    if torch.cuda.is_available():
        torch.cuda.manual_seed_all(seed)
    if deterministic:
        os.environ.setdefault("CUBLAS_WORKSPACE_CONFIG", ":4096:8")
        torch.use_deterministic_algorithms(True, warn_only=True)
    return seed


def get_rng_state() -> dict[str, object]:
    py_version, py_state, py_gauss = random.getstate()
    kind, keys, pos, has_gauss, cached = np.random.get_state()
    state: dict[str, object] = {
        "python": (py_version, tuple(py_state), py_gauss),
        "numpy": {"kind": kind, "keys": torch.from_numpy(np.asarray(keys, dtype=np.int64)),
                  "pos": int(pos), "has_gauss": int(has_gauss), "cached": float(cached)},
        "torch": torch.get_rng_state(),
    }
    if torch.cuda.is_available() and torch.cuda.is_initialized():
        state["cuda"] = torch.cuda.get_rng_state()
    return state


def set_rng_state(state: dict[str, object]) -> None:
    py = state["python"]
    random.setstate((py[0], tuple(py[1]), py[2]))  # type: ignore[index]
    npst = state["numpy"]
    if isinstance(npst, dict):
        keys = np.asarray(npst["keys"].numpy(), dtype=np.uint32)  # type: ignore[union-attr]
        np.random.set_state((npst["kind"], keys, npst["pos"], npst["has_gauss"], npst["cached"]))
    else:  # legacy tuple form
        np.random.set_state(npst)  # type: ignore[arg-type]
    torch.set_rng_state(state["torch"])  # type: ignore[arg-type]
    if "cuda" in state and torch.cuda.is_available():
        torch.cuda.set_rng_state(state["cuda"])  # type: ignore[arg-type]
