"""Lazily zeroed gradient buffers.

The sharding engine does not zero its fp32 gradient buffers at the start of a
step.  It marks every parameter's slice "fresh" instead (contents undefined).
The first kernel that writes a fresh slice overwrites it: the weight-gradient
GEMMs switch their epilogue from accumulate to store, which also saves the
read of the old values.  Kernels that can only accumulate (RMSNorm weight,
embedding rows) zero their slice first.  Before the gradients are reduced the
engine zeroes whatever is still fresh (parameters nobody wrote this step).

A ``main_grad`` view carries ``_dtb_fresh = (FreshSet, offset, numel)``: its
element range in the unit's flat gradient buffer.  Views without the tag
(plain tensors, CPU modules) always accumulate.
"""
from __future__ import annotations

import torch


class FreshSet:
    """Fresh element ranges ``[offset, offset + numel)`` of one flat gradient buffer."""

    def __init__(self, buffer: torch.Tensor) -> None:
        self.buffer = buffer
        self.ranges: dict[int, int] = {}  # offset -> numel

    def mark(self, ranges: list[tuple[int, int]]) -> None:
        self.ranges = dict(ranges)

    def take(self, offset: int, numel: int) -> bool:
        """True (and no longer fresh) when ``[offset, offset+numel)`` is exactly a run of fresh ranges."""
        if offset not in self.ranges:
            self._zero_overlap(offset, numel)
            return False
        end, pos, run = offset + numel, offset, []
        while pos < end and pos in self.ranges:
            run.append(pos)
            pos += self.ranges[pos]
        if pos != end:
            self._zero_overlap(offset, numel)
            return False
        for p in run:
            del self.ranges[p]
        return True

    def _zero_overlap(self, offset: int, numel: int) -> None:
        end = offset + numel
        for p in [p for p, n in self.ranges.items() if p < end and p + n > offset]:
            self.buffer[p:p + self.ranges.pop(p)].zero_()

    def flush(self) -> None:
        """Zero every range nobody wrote."""
        for p, n in self.ranges.items():
            self.buffer[p:p + n].zero_()
        self.ranges.clear()


def tag(view: torch.Tensor, fresh: FreshSet, offset: int) -> torch.Tensor:
    view._dtb_fresh = (fresh, offset, view.numel())  # type: ignore[attr-defined]
    return view


def tag_of(t: torch.Tensor | None):
    return getattr(t, "_dtb_fresh", None) if t is not None else None


def take_fresh(main_grad: torch.Tensor | None) -> bool:
    """Whether the next write into ``main_grad`` may overwrite instead of accumulate."""
    t = tag_of(main_grad)
    return t is not None and t[0].take(t[1], t[2])


def zero_if_fresh(main_grad: torch.Tensor | None) -> None:
    """Make ``main_grad`` safe to accumulate into (zero it if it is still fresh)."""
    if take_fresh(main_grad):
        main_grad.zero_()  # type: ignore[union-attr]
