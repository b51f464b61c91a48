"""Linear layers as autograd functions over the layout-aware GEMMs.

Weight gradients go one of two ways:

* ``main_grad`` given (the sharding engine's fp32 gradient buffer view): the
  weight-grad GEMM accumulates into it in fp32 and autograd receives ``None``
  for the weight — no bf16 gradient tensor is ever allocated, and gradient
  accumulation across micro-steps is the same in-place add.
* no ``main_grad``: a normal gradient tensor is returned (plain modules).

Fused forms: QKV projection with RoPE applied in the GEMM epilogue, and the
gate/up projection with the SwiGLU product in the epilogue.  The reference
runs these as separate cuBLAS GEMMs plus ATen elementwise ops
(``src/model/attention.py:126-131``, ``src/model/mlp.py:72``,
``src/model/embeddings.py:94-114``).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from . import gemm
from .rope import rope_backward_, rope_forward


def _flat(x: torch.Tensor) -> torch.Tensor:
    return x.reshape(-1, x.shape[-1])


def _input_grad(dy2: torch.Tensor, weight: torch.Tensor, grad_comm) -> torch.Tensor:
    if grad_comm is not None:
        return grad_comm.gemm_all_reduce_dgrad(dy2, weight)
    return gemm.mm_nn(dy2, weight)


def _weight_grad(dy2: torch.Tensor, x2: torch.Tensor, weight: torch.Tensor,
                 main_grad: torch.Tensor | None) -> torch.Tensor | None:
    if main_grad is not None:
        gemm.mm_tn_into_grad(dy2, x2, main_grad, weight.shape)
        return None
    if not weight.requires_grad:
        return None
    return gemm.mm_tn(dy2, x2, out_dtype=torch.float32).to(weight.dtype)


class _LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, residual, main_grad):  # type: ignore[override]
        x2 = _flat(x)
        r2 = _flat(residual) if residual is not None else None
        y = gemm.mm_nt(x2, weight.to(x2.dtype) if not x2.is_cuda else weight, residual=r2)
        ctx.save_for_backward(x2, weight)
        ctx.main_grad = main_grad
        ctx.has_res = residual is not None
        return y.view(*x.shape[:-1], weight.shape[0])

    @staticmethod
    def backward(ctx, dy):  # type: ignore[override]
        x2, w = ctx.saved_tensors
        dy2 = _flat(dy).contiguous()
        wc = w if dy2.is_cuda else w.to(dy2.dtype)
        dx = gemm.mm_nn(dy2, wc).view(*dy.shape[:-1], w.shape[1])
        dw = _weight_grad(dy2, x2, w, ctx.main_grad)
        return dx, dw, (dy if ctx.has_res else None), None


def linear(x: torch.Tensor, weight: torch.Tensor, *, bias: torch.Tensor | None = None,
           residual: torch.Tensor | None = None,
           main_grad: torch.Tensor | None = None) -> torch.Tensor:
    """``x @ weight^T (+ bias) (+ residual)``."""
    if not x.is_cuda and main_grad is None:
        y = F.linear(x, weight.to(x.dtype), None if bias is None else bias.to(x.dtype))
        return y + residual if residual is not None else y
    y = _LinearFn.apply(x.contiguous(), weight, residual, main_grad)
    return y + bias if bias is not None else y


def _is_sp(grad_comm) -> bool:
    return getattr(grad_comm, "sp", False)


class _QKVRopeFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, cos, sin, rope_cols, head_dim, seqlen, main_grad, grad_comm):  # type: ignore[override]
        x2 = _flat(x)
        if _is_sp(grad_comm) and head_dim % 64 != 0:
            # no RoPE epilogue for this head size: gather first, then the plain path below
            x2 = grad_comm.comm.all_gather_rows(x2)
        elif _is_sp(grad_comm):
            # x2: this rank's token rows; the GEMM gathers the others' as it goes
            y, x2 = grad_comm.comm.gather_gemm(x2, weight, gemm.EPI_ROPE, cos=cos, sin=sin, p0=rope_cols,
                                               p1=head_dim * 65536 + seqlen)
            ctx.save_for_backward(x2, weight, cos, sin)
            ctx.cfg = (rope_cols, head_dim, seqlen)
            ctx.main_grad = main_grad
            ctx.grad_comm = grad_comm
            return y
        if x2.is_cuda and head_dim % 64 == 0:
            y = gemm.mm_nt_rope(x2, weight, cos, sin, rope_cols, head_dim, seqlen)
        elif x2.is_cuda:  # head sizes the RoPE epilogue does not tile: GEMM, then the RoPE kernel
            y = gemm.mm_nt(x2, weight)
            rope_forward(y, cos, sin, rope_cols, head_dim, seqlen)
        else:
            y = gemm.mm_nt(x2, weight.to(x2.dtype))
            rope_forward(y, cos, sin, rope_cols, head_dim, seqlen)
        ctx.save_for_backward(x2, weight, cos, sin)
        ctx.cfg = (rope_cols, head_dim, seqlen)
        ctx.main_grad = main_grad
        ctx.grad_comm = grad_comm
        return y.view(*x.shape[:-1], weight.shape[0])

    @staticmethod
    def backward(ctx, dy):  # type: ignore[override]
        x2, w, cos, sin = ctx.saved_tensors
        rope_cols, head_dim, seqlen = ctx.cfg
        d = _flat(dy).contiguous().clone()
        rope_backward_(d, cos, sin, rope_cols, head_dim, seqlen)
        wc = w if d.is_cuda else w.to(d.dtype)
        if _is_sp(ctx.grad_comm):
            dx = ctx.grad_comm.comm.dgrad_reduce_scatter(d, wc)
        else:
            dx = _input_grad(d, wc, ctx.grad_comm).view(*dy.shape[:-1], w.shape[1])
        dw = _weight_grad(d, x2, w, ctx.main_grad)
        return dx, dw, None, None, None, None, None, None, None


def linear_qkv_rope(x: torch.Tensor, weight: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                    n_q_heads: int, n_kv_heads: int, head_dim: int, seqlen: int, *,
                    main_grad: torch.Tensor | None = None, grad_comm=None) -> torch.Tensor:
    """Packed ``[q | k | v]`` projection with RoPE applied to ``q`` and ``k``.

    ``weight`` is ``[Wq; Wk; Wv]`` (``[(nq + 2 nkv) * hd, d]``); ``x`` is
    ``[b, s, d]`` or ``[b*s, d]`` with token ``m`` at position ``m % seqlen``.
    """
    rope_cols = (n_q_heads + n_kv_heads) * head_dim
    return _QKVRopeFn.apply(x.contiguous(), weight, cos, sin, rope_cols, head_dim, seqlen,
                            main_grad, grad_comm)


def swiglu_reference(gu: torch.Tensor, ffn: int) -> torch.Tensor:
    g, u = gu[..., :ffn], gu[..., ffn:]
    return F.silu(g) * u


def swiglu_backward(dact: torch.Tensor, gu: torch.Tensor, ffn: int) -> torch.Tensor:
    """``d[g|u]`` from ``d(silu(g) * u)``; fp32 math, output in ``gu``'s dtype."""
    if dact.is_cuda:
        from ._ext import native
        out = torch.empty_like(gu)
        native().swiglu_bwd(dact.contiguous(), gu, out)
        return out
    g, u = gu[..., :ffn].float(), gu[..., ffn:].float()
    sg = torch.sigmoid(g)
    silu = g * sg
    da = dact.float()
    dg = da * u * (sg * (1 + g * (1 - sg)))
    du = da * silu
    return torch.cat([dg, du], dim=-1).to(gu.dtype)


class _SwiGLUFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, ffn, main_grad, grad_comm):  # type: ignore[override]
        x2 = _flat(x)
        if _is_sp(grad_comm) and ffn % 128 == 0:
            (act, gu), x2 = grad_comm.comm.gather_gemm(x2, weight, gemm.EPI_SWIGLU, ffn=ffn)
            ctx.save_for_backward(x2, weight, gu)
            ctx.ffn = ffn
            ctx.main_grad = main_grad
            ctx.grad_comm = grad_comm
            return act
        if _is_sp(grad_comm):  # no SwiGLU epilogue for this width: gather first, then the plain path
            x2 = grad_comm.comm.all_gather_rows(x2)
        if x2.is_cuda and ffn % 128 == 0:
            act, gu = gemm.mm_nt_swiglu(x2, weight, ffn)
        else:
            gu = gemm.mm_nt(x2, weight if x2.is_cuda else weight.to(x2.dtype))
            act = swiglu_reference(gu, ffn)
            if x2.is_cuda:
                act = act.contiguous()
        ctx.save_for_backward(x2, weight, gu)
        ctx.ffn = ffn
        ctx.main_grad = main_grad
        ctx.grad_comm = grad_comm
        return act.view(*x.shape[:-1], ffn)

    @staticmethod
    def backward(ctx, dact):  # type: ignore[override]
        x2, w, gu = ctx.saved_tensors
        dgu = swiglu_backward(_flat(dact), gu, ctx.ffn)
        wc = w if dgu.is_cuda else w.to(dgu.dtype)
        if _is_sp(ctx.grad_comm):
            dx = ctx.grad_comm.comm.dgrad_reduce_scatter(dgu, wc)
        else:
            dx = _input_grad(dgu, wc, ctx.grad_comm).view(*dact.shape[:-1], w.shape[1])
        dw = _weight_grad(dgu, x2, w, ctx.main_grad)
        return dx, dw, None, None, None


def linear_swiglu(x: torch.Tensor, weight: torch.Tensor, ffn: int, *,
                  main_grad: torch.Tensor | None = None, grad_comm=None) -> torch.Tensor:
    """``silu(x W_g^T) * (x W_u^T)`` with ``weight = [W_g; W_u]`` (``[2F, d]``).

    ``grad_comm``: a TP transport whose ``gemm_all_reduce_dgrad`` computes the
    input gradient and its TP all-reduce in one kernel (column-parallel use).
    """
    return _SwiGLUFn.apply(x.contiguous(), weight, ffn, main_grad, grad_comm)
