"""RMSNorm: ``y = x * rsqrt(mean(x^2) + eps) * w`` with fp32 statistics.

Reference math: ``src/model/transformer.py:63-68``.  On CUDA one kernel reads
``x`` once and writes ``y`` plus the per-row ``rstd`` it saves for backward;
the backward kernel produces ``dx`` and accumulates ``dw`` in fp32 in a fixed
order (deterministic; into the engine's ``main_grad`` when given).
"""

from __future__ import annotations

import torch

from . import grad_state
from ._ext import native


def rms_norm_reference(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    dt = x.dtype
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return y.to(dt) * weight.to(dt)


class _RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, eps, main_grad):  # type: ignore[override]
        x2 = x.reshape(-1, x.shape[-1])
        if x2.is_cuda:
            y, rstd = native().rmsnorm_fwd(x2, weight, eps)
        else:
            xf = x2.float()
            rstd = torch.rsqrt(xf.pow(2).mean(-1) + eps)
            y = ((xf * rstd[:, None]) * weight.float()).to(x2.dtype)
        ctx.save_for_backward(x2, weight, rstd)
        ctx.main_grad = main_grad
        return y.view_as(x)

    @staticmethod
    def backward(ctx, dy):  # type: ignore[override]
        x2, w, rstd = ctx.saved_tensors
        dy2 = dy.reshape(-1, dy.shape[-1]).contiguous()
        mg = ctx.main_grad
        grad_state.zero_if_fresh(mg)  # the dw reduction accumulates
        if dy2.is_cuda:
            acc = mg if mg is not None else torch.zeros(w.shape, device=w.device, dtype=torch.float32)
            dx = native().rmsnorm_bwd(dy2, x2, w, rstd, acc)
            dw = None if mg is not None else acc.to(w.dtype)
        else:
            xf, g = x2.float(), dy2.float()
            xhat = xf * rstd[:, None]
            gw = g * w.float()
            dx = (rstd[:, None] * (gw - xhat * (gw * xhat).mean(-1, keepdim=True))).to(x2.dtype)
            dwf = (g * xhat).sum(0)
            if mg is not None:
                mg.add_(dwf)
                dw = None
            else:
                dw = dwf.to(w.dtype)
        return dx.view_as(dy), dw, None, None


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float, *,
             main_grad: torch.Tensor | None = None) -> torch.Tensor:
    if not x.is_cuda and main_grad is None:
        return rms_norm_reference(x, weight, eps)
    return _RMSNormFn.apply(x.contiguous(), weight, eps, main_grad)
