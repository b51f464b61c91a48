"""Causal grouped-query attention over the packed ``[q | k | v]`` projection.

The CPU path restates the reference (``src/model/attention.py:109-155``):
``repeat_kv`` then ``scaled_dot_product_attention(is_causal=True)``.  The CUDA
path is the flash-attention kernel pair of ``csrc/attention.cu``: it reads
q/k/v straight out of the packed projection (no transposes, no ``repeat_kv``
copy: a query head ``h`` reads kv head ``h // (nq/nkv)``), keeps the running
softmax in registers, writes ``o`` as ``[b*s, nq*hd]`` (the layout the output
projection consumes) and saves only the per-row log-sum-exp for backward.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from ._ext import native


def repeat_kv(x: torch.Tensor, n_rep: int) -> torch.Tensor:
    """``[b, s, kv, d] -> [b, s, kv * n_rep, d]``, each kv head repeated ``n_rep`` times."""
    if n_rep == 1:
        return x
    b, s, kv, d = x.shape
    return x[:, :, :, None, :].expand(b, s, kv, n_rep, d).reshape(b, s, kv * n_rep, d)


def attention_reference(qkv: torch.Tensor, batch: int, seqlen: int, nq: int, nkv: int,
                        hd: int, dropout_p: float = 0.0) -> torch.Tensor:
    q = qkv[..., : nq * hd].reshape(batch, seqlen, nq, hd)
    k = qkv[..., nq * hd:(nq + nkv) * hd].reshape(batch, seqlen, nkv, hd)
    v = qkv[..., (nq + nkv) * hd:].reshape(batch, seqlen, nkv, hd)
    k, v = repeat_kv(k, nq // nkv), repeat_kv(v, nq // nkv)
    o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                       is_causal=True, dropout_p=dropout_p)
    return o.transpose(1, 2).reshape(batch * seqlen, nq * hd)


# head sizes with a native kernel: tcgen05/TMEM for 64 and 128 at seq_len % 128 == 0,
# mma.sync for the rest (any seq_len)
KERNEL_HEAD_DIMS = (16, 32, 64, 128)


class _FlashAttnFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, batch, seqlen, nq, nkv, hd):  # type: ignore[override]
        scale = 1.0 / math.sqrt(hd)
        o, lse = native().attn_fwd(qkv, batch, seqlen, nq, nkv, hd, scale)
        ctx.save_for_backward(qkv, o, lse)
        ctx.cfg = (batch, seqlen, nq, nkv, hd, scale)
        return o

    @staticmethod
    def backward(ctx, do):  # type: ignore[override]
        qkv, o, lse = ctx.saved_tensors
        b, s, nq, nkv, hd, scale = ctx.cfg
        dqkv = native().attn_bwd(do.contiguous(), qkv, o, lse, b, s, nq, nkv, hd, scale)
        return dqkv, None, None, None, None, None


def causal_attention(qkv: torch.Tensor, batch: int, seqlen: int, n_q_heads: int,
                     n_kv_heads: int, head_dim: int, dropout_p: float = 0.0) -> torch.Tensor:
    """``qkv: [b*s, (nq + 2 nkv) * hd]`` -> ``o: [b*s, nq * hd]``."""
    if n_q_heads % n_kv_heads:
        raise ValueError(f"{n_q_heads} query heads are not a multiple of {n_kv_heads} kv heads")
    if not qkv.is_cuda or dropout_p > 0.0 or head_dim not in KERNEL_HEAD_DIMS:
        # attention dropout (the shipped configs train with 0.0) and head sizes without a
        # kernel run PyTorch's SDPA, the reference's own kernel (src/model/attention.py:147)
        return attention_reference(qkv, batch, seqlen, n_q_heads, n_kv_heads, head_dim, dropout_p)
    return _FlashAttnFn.apply(qkv.contiguous(), batch, seqlen, n_q_heads, n_kv_heads, head_dim)
