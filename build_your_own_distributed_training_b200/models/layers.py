"""Parameter containers shared by the model modules.

``Linear`` holds ``weight [out, in]`` (+ optional ``bias``) under the same
names as ``nn.Linear`` so checkpoint keys match the reference's
(``layers.{i}.attention.wq.weight`` and so on).  It carries no forward of its
own: the blocks call the fused ops directly, which lets two or three adjacent
weights be consumed by one GEMM.

``fused_rows`` returns the row-concatenation of several weights: a zero-copy
view when they are adjacent in memory and the sharding engine owns their
gradients (``main_grad``), otherwise a differentiable ``torch.cat``.
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn

from ..ops import grad_state


class Linear(nn.Module):
    def __init__(self, in_features: int, out_features: int, bias: bool = False) -> None:
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        self.weight = nn.Parameter(torch.empty(out_features, in_features))
        self.bias = nn.Parameter(torch.zeros(out_features)) if bias else None
        nn.init.kaiming_uniform_(self.weight, a=math.sqrt(5))

    def extra_repr(self) -> str:
        return f"in_features={self.in_features}, out_features={self.out_features}, bias={self.bias is not None}"


def _adjacent_view(ts: list[torch.Tensor]) -> torch.Tensor | None:
    base = ts[0]
    ptr = base.untyped_storage().data_ptr()
    off = base.storage_offset()
    for t in ts:
        if (t.untyped_storage().data_ptr() != ptr or t.storage_offset() != off
                or not t.is_contiguous()):
            return None
        off += t.numel()
    rows = sum(t.shape[0] for t in ts)
    cols = base.shape[1] if base.dim() == 2 else 1
    return base.detach().as_strided((rows, cols), (cols, 1), base.storage_offset())


def fused_rows(params: list[torch.Tensor]) -> tuple[torch.Tensor, torch.Tensor | None]:
    """``(W, main_grad)`` for the row-stack of ``params``."""
    grads = [getattr(p, "main_grad", None) for p in params]
    if all(g is not None for g in grads):
        w = _adjacent_view(params)
        mg = _adjacent_view(grads)  # type: ignore[arg-type]
        if w is not None and mg is not None:
            first = grad_state.tag_of(grads[0])
            if first is not None:  # the stacked view covers the constituents' fresh ranges
                grad_state.tag(mg, first[0], first[1])
            return w, mg
    if len(params) == 1:
        return params[0], grads[0]
    return torch.cat(params, dim=0), None


def main_grad_of(p: torch.Tensor) -> torch.Tensor | None:
    return getattr(p, "main_grad", None)
