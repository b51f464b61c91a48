"""Dtype names and the mixed-precision policy.

Policy (same meaning as the FSDP ``MixedPrecision`` the reference builds in
``src/utils/dtype.py:74-106``): compute parameters are ``param_dtype``
(bf16 on GPU), gradients are reduced in ``reduce_dtype`` (fp32) and the
optimizer owns an fp32 master copy.  Here the policy is a plain record that
the sharding engine reads; there is no FSDP wrapper.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

_NAMES: dict[str, torch.dtype] = {
    "float32": torch.float32, "fp32": torch.float32, "float": torch.float32,
    "float16": torch.float16, "fp16": torch.float16, "half": torch.float16,
    "bfloat16": torch.bfloat16, "bf16": torch.bfloat16,
}


def resolve_dtype(name: str) -> torch.dtype:
    key = name.strip().lower()
    if key not in _NAMES:
        raise ValueError(f"Unknown dtype {name!r}; valid names: {sorted(_NAMES)}.")
    return _NAMES[key]


@dataclass(frozen=True)
class MixedPrecisionPolicy:
    param_dtype: torch.dtype
    reduce_dtype: torch.dtype
    buffer_dtype: torch.dtype
    master_dtype: torch.dtype = torch.float32


def build_mixed_precision(cfg) -> MixedPrecisionPolicy:  # cfg: ParallelConfig
    return MixedPrecisionPolicy(resolve_dtype(cfg.param_dtype), resolve_dtype(cfg.reduce_dtype),
                                resolve_dtype(cfg.buffer_dtype))


def autocast_dtype(cfg) -> torch.dtype:
    """Compute dtype of the forward (the parameter dtype)."""
    return resolve_dtype(cfg.param_dtype)
