"""Token embedding gather with a deterministic backward.

Forward: row gather.  Backward on CUDA: token ids are sorted, then each block
sums the incoming gradient rows of one token id in sorted order and adds the
sum to the fp32 gradient (``main_grad`` when given).  Every run therefore
produces the same bits, which bit-exact resume relies on; the reference used
ATen's ``embedding_backward`` (``src/model/embeddings.py:53``).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from . import grad_state
from ._ext import native


class _EmbeddingFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, tokens, weight, main_grad, out_dtype):  # type: ignore[override]
        if weight.is_cuda:
            out = native().embedding_fwd(tokens.reshape(-1).contiguous(), weight, out_dtype)
        else:
            out = F.embedding(tokens.reshape(-1), weight).to(out_dtype)
        ctx.save_for_backward(tokens)
        ctx.main_grad = main_grad
        ctx.wshape = weight.shape
        ctx.wdtype = weight.dtype
        ctx.requires_w = weight.requires_grad
        return out.view(*tokens.shape, weight.shape[1])

    @staticmethod
    def backward(ctx, dout):  # type: ignore[override]
        (tokens,) = ctx.saved_tensors
        mg = ctx.main_grad
        grad_state.zero_if_fresh(mg)  # rows are scatter-added
        acc = mg.view(ctx.wshape) if mg is not None else torch.zeros(
            ctx.wshape, device=dout.device, dtype=torch.float32)
        if dout.is_cuda:
            native().embedding_bwd(tokens.reshape(-1).contiguous(),
                                   dout.reshape(-1, ctx.wshape[1]).contiguous(), acc)
        else:
            acc.index_add_(0, tokens.reshape(-1), dout.reshape(-1, ctx.wshape[1]).float())
        if mg is not None or not ctx.requires_w:
            return None, None, None, None
        return None, acc.to(ctx.wdtype), None, None


def embedding(tokens: torch.Tensor, weight: torch.Tensor, *, main_grad: torch.Tensor | None = None,
              out_dtype: torch.dtype | None = None) -> torch.Tensor:
    if not weight.is_cuda and main_grad is None:
        out = F.embedding(tokens, weight)
        return out if out_dtype is None else out.to(out_dtype)
    return _EmbeddingFn.apply(tokens, weight, main_grad, out_dtype or weight.dtype)
