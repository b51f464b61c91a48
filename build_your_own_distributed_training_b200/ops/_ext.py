"""Loader for the native extension ``_C`` (sm_100a kernels + C++ runtime).

The extension is built in-tree by ``setup.py build_ext --inplace``.  On a CUDA
tensor every op calls into it; if it is missing the op raises instead of
falling back to PyTorch, so a run can never silently measure library code.
"""

from __future__ import annotations

import importlib

_mod = None
_err: Exception | None = None


def native():
    """Return the ``_C`` module or raise with the build hint."""
    global _mod, _err
    if _mod is None and _err is None:
        try:
            _mod = importlib.import_module("build_your_own_distributed_training_b200._C")
        except Exception as exc:  # noqa: BLE001
            _err = exc
    if _mod is None:
        raise RuntimeError(
            "native extension build_your_own_distributed_training_b200._C is not built "
            f"({_err!r}); run `python setup.py build_ext --inplace` at the repo root."
        )
    return _mod


def available() -> bool:
    try:
        native()
        return True
    except RuntimeError:
        return False
