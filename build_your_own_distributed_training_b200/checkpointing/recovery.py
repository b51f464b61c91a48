"""Checkpoint validation and newest-valid discovery (``src/checkpointing/recovery.py:39-209``).

``validate_checkpoint`` checks the marker, ``meta.json``, every rank's
``model.pt`` (present, non-empty, loadable when ``deep``), the full-format file
and the model-config keys that make a checkpoint incompatible.
"""

from __future__ import annotations

import json
import os
from dataclasses import dataclass, field
from typing import Any

from .checkpoint import META_FILE, SUCCESS_MARKER, safe_load

MODEL_CONFIG_KEYS = ("vocab_size", "d_model", "n_layers", "n_heads", "n_kv_heads",
                     "ffn_hidden_size", "max_seq_len")


class CheckpointValidationError(Exception):
    pass


@dataclass
class CheckpointValidationResult:
    path: str
    is_valid: bool
    step: int = -1
    world_size: int = -1
    errors: list[str] = field(default_factory=list)


def _deep_check(path: str, errors: list[str]) -> None:
    try:
        safe_load(path)
    except Exception as exc:  # noqa: BLE001 - any load failure makes the shard corrupt
        errors.append(f"corrupt/unloadable shard {path}: {exc!r}")


def _check_file(path: str, label: str, deep: bool, errors: list[str]) -> None:
    if not os.path.exists(path):
        errors.append(f"missing {label}: {path}")
    elif os.path.getsize(path) == 0:
        errors.append(f"zero-byte {label}: {path}")
    elif deep:
        _deep_check(path, errors)


def validate_checkpoint(path: str, *, expected_config: dict[str, Any] | None = None,
                        deep: bool = False) -> CheckpointValidationResult:
    errors: list[str] = []
    if not os.path.isdir(path):
        return CheckpointValidationResult(path, False, errors=[f"not a directory: {path}"])
    if not os.path.exists(os.path.join(path, SUCCESS_MARKER)):
        errors.append(f"missing {SUCCESS_MARKER} marker (save incomplete)")
    meta: dict[str, Any] = {}
    step = world = -1
    mpath = os.path.join(path, META_FILE)
    if not os.path.exists(mpath):
        errors.append(f"missing {META_FILE}")
    else:
        try:
            with open(mpath) as f:
                meta = json.load(f)
            step, world = int(meta.get("step", -1)), int(meta.get("world_size", -1))
        except (json.JSONDecodeError, ValueError) as exc:
            errors.append(f"unreadable {META_FILE}: {exc}")
    fmt = meta.get("format", "sharded")
    if fmt == "sharded" and world > 0:
        for r in range(world):
            _check_file(os.path.join(path, f"rank_{r}", "model.pt"), f"shard for rank {r}", deep, errors)
    elif fmt == "full":
        _check_file(os.path.join(path, "model_full.pt"), "model_full.pt", deep, errors)
    if expected_config is not None and meta.get("config"):
        saved = meta["config"].get("model", {})
        want = expected_config.get("model", {})
        for k in MODEL_CONFIG_KEYS:
            a, b = want.get(k), saved.get(k)
            if a is not None and b is not None and a != b:
                errors.append(f"model config mismatch on {k!r}: checkpoint={b} current={a}")
    return CheckpointValidationResult(path, not errors, step, world, errors)


def find_latest_valid_checkpoint(checkpoint_dir: str, *, expected_config: dict[str, Any] | None = None,
                                 deep: bool = False) -> str | None:
    if not os.path.isdir(checkpoint_dir):
        return None
    steps = []
    for name in os.listdir(checkpoint_dir):
        if name.startswith("step_"):
            try:
                steps.append((int(name[5:]), os.path.join(checkpoint_dir, name)))
            except ValueError:
                continue
    for _, p in sorted(steps, reverse=True):
        if validate_checkpoint(p, expected_config=expected_config, deep=deep).is_valid:
            return p
    return None


def require_valid_checkpoint(path: str, *, expected_config: dict[str, Any] | None = None,
                             deep: bool = True) -> CheckpointValidationResult:
    res = validate_checkpoint(path, expected_config=expected_config, deep=deep)
    if not res.is_valid:
        raise CheckpointValidationError(f"Checkpoint {path} is invalid:\n  - " + "\n  - ".join(res.errors))
    return res
