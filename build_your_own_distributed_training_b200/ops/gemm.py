"""GEMM entry points in the three layouts a linear layer needs.

``C[M,N] = sum_k A(m,k) B(n,k)`` with each operand either K-major (the
reduction axis is contiguous) or MN-major.  A linear layer ``y = x W^T`` with
``x:[M,K]`` and ``W:[N,K]`` uses

* forward ``mm_nt(x, W)``: both K-major;
* input grad ``mm_nn(dy, W)``: ``dy`` K-major, ``W`` MN-major (no transpose copy);
* weight grad ``mm_tn_acc(dy, x, acc)``: both MN-major, fp32 accumulated in place
  into the sharding engine's gradient buffer.

On CUDA these run the tcgen05 kernel of ``csrc/gemm.cu``; on CPU they are
``torch.matmul`` in the input dtype (the oracle).
"""

from __future__ import annotations

import torch

from . import grad_state
from ._ext import native

# epilogue codes shared with csrc/gemm.cu
EPI_STORE = 0        # D = acc (D's dtype: bf16 or fp32)
EPI_ACC_F32 = 2      # D(fp32) += acc
EPI_RESIDUAL = 3     # D = acc + R
EPI_ROPE = 4         # D = acc with rotate-half RoPE on the first p0 columns, heads of p1
EPI_SWIGLU = 5       # D = silu(g) * u ; D2 = [g | u]  (g, u: 128-column tiles of B rows n and n+p0)
EPI_ACC_BF16OUT = 9  # D(bf16) = acc + R(fp32)  (last step of a GEMM chunked over K)


def _check_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if t is not None and not t.is_contiguous():
            raise ValueError("GEMM operands must be contiguous")


def mm_nt(a: torch.Tensor, b: torch.Tensor, *, residual: torch.Tensor | None = None,
          out_dtype: torch.dtype | None = None, alpha: torch.Tensor | None = None,
          out: torch.Tensor | None = None) -> torch.Tensor:
    """``a[M,K] @ b[N,K]^T`` (+ ``residual``)."""
    M, N = a.shape[0], b.shape[0]
    if not a.is_cuda:
        y = a @ b.t()
        if alpha is not None:
            y = y * alpha
        if residual is not None:
            y = y + residual
        return y.to(out_dtype) if out_dtype is not None else y
    _check_cuda(a, b, residual)
    dt = out_dtype or a.dtype
    if out is None:
        out = torch.empty(M, N, device=a.device, dtype=dt)
    epi = EPI_RESIDUAL if residual is not None else EPI_STORE
    native().gemm(a, b, out, False, False, epi, residual, alpha, None, None, None, 0, 0)
    return out


def mm_nn(a: torch.Tensor, b: torch.Tensor, *, alpha: torch.Tensor | None = None,
          out: torch.Tensor | None = None) -> torch.Tensor:
    """``a[M,K] @ b[K,N]``."""
    if not a.is_cuda:
        y = a @ b
        return y * alpha if alpha is not None else y
    _check_cuda(a, b)
    if out is None:
        out = torch.empty(a.shape[0], b.shape[1], device=a.device, dtype=a.dtype)
    native().gemm(a, b, out, False, True, EPI_STORE, None, alpha, None, None, None, 0, 0)
    return out


def mm_tn_acc(a: torch.Tensor, b: torch.Tensor, acc: torch.Tensor, *,
              alpha: torch.Tensor | None = None, store: bool = False) -> torch.Tensor:
    """``acc[M,N] += a[K,M]^T @ b[K,N]`` with ``acc`` fp32 (weight gradients); ``store`` overwrites."""
    if not a.is_cuda:
        y = a.t().to(acc.dtype) @ b.to(acc.dtype)
        y = y * alpha if alpha is not None else y
        acc.copy_(y) if store else acc.add_(y)
        return acc
    _check_cuda(a, b, acc)
    if acc.dtype != torch.float32:
        raise ValueError("mm_tn_acc accumulates into an fp32 buffer")
    native().gemm(a, b, acc, True, True, EPI_STORE if store else EPI_ACC_F32, None, alpha, None, None, None, 0, 0)
    return acc


def mm_tn_into_grad(a: torch.Tensor, b: torch.Tensor, main_grad: torch.Tensor, shape, *,
                    alpha: torch.Tensor | None = None) -> torch.Tensor:
    """Weight gradient ``a^T b`` into a gradient slice: overwritten while the slice is
    fresh (first writer of the step), accumulated afterwards."""
    store = grad_state.take_fresh(main_grad)
    return mm_tn_acc(a, b, main_grad.view(shape), alpha=alpha, store=store)


def mm_tn(a: torch.Tensor, b: torch.Tensor, *, alpha: torch.Tensor | None = None,
          out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """``a[K,M]^T @ b[K,N]`` into a fresh tensor."""
    if not a.is_cuda:
        y = a.t().float() @ b.float()
        y = y * alpha if alpha is not None else y
        return y.to(out_dtype)
    out = torch.empty(a.shape[1], b.shape[1], device=a.device, dtype=out_dtype)
    native().gemm(a, b, out, True, True, EPI_STORE, None, alpha, None, None, None, 0, 0)
    return out


def mm_nt_rope(a: torch.Tensor, b: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
               rope_cols: int, head_dim: int, seqlen: int) -> torch.Tensor:
    """``a @ b^T`` with rotate-half RoPE applied to output columns ``< rope_cols``.

    Row ``m`` of ``a`` is token position ``m % seqlen``; ``cos``/``sin`` are
    fp32 ``[>=seqlen, head_dim]`` tables.
    """
    out = torch.empty(a.shape[0], b.shape[0], device=a.device, dtype=a.dtype)
    native().gemm(a, b, out, False, False, EPI_ROPE, None, None, cos, sin, None,
                  rope_cols, head_dim * 65536 + seqlen)
    return out


def mm_nt_swiglu(a: torch.Tensor, b: torch.Tensor, ffn: int) -> tuple[torch.Tensor, torch.Tensor]:
    """``b = [W_gate; W_up]`` (``[2F, K]``): returns ``silu(a W_g^T) * (a W_u^T)`` and ``[g|u]``."""
    M = a.shape[0]
    act = torch.empty(M, ffn, device=a.device, dtype=a.dtype)
    gu = torch.empty(M, 2 * ffn, device=a.device, dtype=a.dtype)
    native().gemm(a, b, act, False, False, EPI_SWIGLU, None, None, None, None, gu, ffn, 0)
    return act, gu
