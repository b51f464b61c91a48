"""LM head + cross-entropy (mean over labels != -100).

Reference: ``src/model/transformer.py:184-191`` (cuBLAS GEMM to logits, then
``F.cross_entropy`` in fp32).  CUDA path: the tcgen05 GEMM writes fp32 logits,
one kernel per row computes the log-sum-exp, the loss contribution and the
bf16 logit gradient ``(softmax - onehot) / n_valid`` in the same pass, and the
backward is two GEMMs scaled by the incoming gradient read from device memory
(no host sync).  The head weight gradient accumulates into ``main_grad``
(shared with the embedding when the weights are tied).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from . import gemm
from ._ext import native


class _HeadCEFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, w, labels, main_grad, keep_logits):  # type: ignore[override]
        logits = gemm.mm_nt(h, w, out_dtype=torch.float32)
        loss, dlogits = native().cross_entropy_fwd(logits, labels, -100)
        ctx.save_for_backward(h, w, dlogits)
        ctx.main_grad = main_grad
        return loss, (logits if keep_logits else None)

    @staticmethod
    def backward(ctx, dloss, _dlogits_unused):  # type: ignore[override]
        h, w, dlogits = ctx.saved_tensors
        alpha = dloss.reshape(1).float().contiguous()
        dh = gemm.mm_nn(dlogits, w, alpha=alpha)
        if ctx.main_grad is not None:
            gemm.mm_tn_into_grad(dlogits, h, ctx.main_grad, w.shape, alpha=alpha)
            dw = None
        elif w.requires_grad:
            dw = gemm.mm_tn(dlogits, h, alpha=alpha).to(w.dtype)
        else:
            dw = None
        return dh, dw, None, None, None


def lm_head_cross_entropy(h: torch.Tensor, weight: torch.Tensor, labels: torch.Tensor | None, *,
                          main_grad: torch.Tensor | None = None, return_logits: bool = True
                          ) -> tuple[torch.Tensor | None, torch.Tensor | None]:
    """Returns ``(logits or None, loss or None)`` for ``h: [M, d]``, ``labels: [M]``."""
    if not h.is_cuda or labels is None:
        from .linear import linear
        logits = linear(h, weight, main_grad=main_grad)
        loss = None
        if labels is not None:
            loss = F.cross_entropy(logits.float(), labels.reshape(-1), ignore_index=-100)
        return logits, loss
    loss, logits = _HeadCEFn.apply(h.contiguous(), weight, labels.reshape(-1).contiguous(),
                                   main_grad, return_logits)
    return logits, loss
