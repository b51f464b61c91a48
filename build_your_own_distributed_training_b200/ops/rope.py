"""Rotary position embedding in the rotate-half layout.

Cache: ``cos/sin[pos, j]`` fp32 of shape ``(max_seq, head_dim)`` with the
frequency table duplicated across the two halves, so element ``j`` pairs with
``j + head_dim/2`` (reference ``src/model/embeddings.py:56-114``).

On CUDA the forward rotation happens inside the QKV GEMM epilogue; the
backward (the transposed rotation) is the ``rope_bwd`` kernel applied to the
packed ``[dq | dk | dv]`` gradient in place.
"""

from __future__ import annotations

import torch


def precompute_rope_cache(head_dim: int, max_seq_len: int, theta: float,
                          device: torch.device | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    if head_dim % 2:
        raise ValueError(f"RoPE needs an even head_dim, got {head_dim}.")
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, device=device).float() / head_dim))
    ang = torch.outer(torch.arange(max_seq_len, device=device).float(), inv_freq)
    ang = torch.cat((ang, ang), dim=-1)
    return ang.cos(), ang.sin()


def _rotate_half(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


def apply_rotary_emb(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate ``x:[b, s, h, d]`` with cache slices ``[s, d]`` (computed in ``x``'s dtype)."""
    c = cos[None, :, None, :].to(x.dtype)
    s = sin[None, :, None, :].to(x.dtype)
    return x * c + _rotate_half(x) * s


def _heads_view(y: torch.Tensor, rope_cols: int, head_dim: int, seqlen: int) -> torch.Tensor:
    M = y.shape[0]
    return y[:, :rope_cols].reshape(M // seqlen, seqlen, rope_cols // head_dim, head_dim)


def rope_forward(y: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, rope_cols: int,
                 head_dim: int, seqlen: int) -> None:
    """In place on a packed 2-D ``[b*s, cols]`` tensor, first ``rope_cols`` columns."""
    if y.is_cuda and y.dtype == torch.bfloat16:
        from ._ext import native
        native().rope_fwd(y, cos, sin, rope_cols, head_dim, seqlen)
        return
    v = _heads_view(y, rope_cols, head_dim, seqlen)
    c, s = cos[:seqlen][None, :, None, :], sin[:seqlen][None, :, None, :]
    rot = (v.float() * c + _rotate_half(v.float()) * s).to(y.dtype)
    y[:, :rope_cols] = rot.reshape(y.shape[0], rope_cols)


def rope_backward_(d: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, rope_cols: int,
                   head_dim: int, seqlen: int) -> None:
    """Apply the transposed rotation in place (gradient of :func:`rope_forward`)."""
    if d.is_cuda:
        from ._ext import native
        native().rope_bwd(d, cos, sin, rope_cols, head_dim, seqlen)
        return
    v = _heads_view(d, rope_cols, head_dim, seqlen).float()
    c, s = cos[:seqlen][None, :, None, :], sin[:seqlen][None, :, None, :]
    h = head_dim // 2
    vs = v * s
    back = v * c + torch.cat((vs[..., h:], -vs[..., :h]), dim=-1)
    d[:, :rope_cols] = back.to(d.dtype).reshape(d.shape[0], rope_cols)
