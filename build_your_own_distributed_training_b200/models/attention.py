"""Causal grouped-query attention block (reference ``src/model/attention.py:70-155``).

Parameters keep the reference names ``wq, wk, wv, wo``.  The forward runs
three fused ops: the packed QKV projection with RoPE in its epilogue, flash
attention reading the packed buffer (local head counts are inferred from the
possibly TP-sharded weight shapes, as the reference's ``view(..., -1, hd)``
did), and the output projection with the residual add fused (and, under TP,
the all-reduce or reduce-scatter fused with it).
"""

from __future__ import annotations

import torch
import torch.nn as nn

from ..config import ModelConfig
from ..ops.attention import causal_attention, repeat_kv  # noqa: F401
from ..ops.linear import linear_qkv_rope
from ..parallel import tensor_parallel as tpar
from .layers import Linear, fused_rows, main_grad_of


class Attention(nn.Module):
    def __init__(self, config: ModelConfig) -> None:
        super().__init__()
        assert config.n_kv_heads is not None
        self.n_heads = config.n_heads
        self.n_kv_heads = config.n_kv_heads
        self.head_dim = config.head_dim
        self.dropout_p = config.dropout
        kv = self.n_kv_heads * self.head_dim
        self.wq = Linear(config.d_model, config.d_model, config.attention_bias)
        self.wk = Linear(config.d_model, kv, config.attention_bias)
        self.wv = Linear(config.d_model, kv, config.attention_bias)
        self.wo = Linear(config.d_model, config.d_model, config.attention_bias)
        self.tp: tpar.TPInfo | None = None

    def forward(self, x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                residual: torch.Tensor | None = None) -> torch.Tensor:
        """``x``: ``[b, s, d]`` (or local ``[tokens, d]`` under sequence parallelism)."""
        out_shape = x.shape if residual is None else residual.shape
        seqlen = cos.shape[0]
        # under sequence parallelism x2 may stay this rank's rows: the QKV GEMM gathers them
        x2, grad_comm = tpar.column_input_fused(x.reshape(-1, x.shape[-1]), self.tp,
                                                sp_ok=self.wq.bias is None)
        hd = self.head_dim
        nq, nkv = self.wq.weight.shape[0] // hd, self.wk.weight.shape[0] // hd
        if self.wq.bias is not None:
            w = torch.cat([self.wq.weight, self.wk.weight, self.wv.weight])
            b = torch.cat([self.wq.bias, self.wk.bias, self.wv.bias])
            qkv = torch.nn.functional.linear(x2, w.to(x2.dtype), b.to(x2.dtype))
            from ..ops.rope import rope_forward
            qkv = qkv.clone()
            rope_forward(qkv, cos, sin, (nq + nkv) * hd, hd, seqlen)
        else:
            w, mg = fused_rows([self.wq.weight, self.wk.weight, self.wv.weight])
            qkv = linear_qkv_rope(x2, w, cos, sin, nq, nkv, hd, seqlen, main_grad=mg, grad_comm=grad_comm)
        o = causal_attention(qkv, qkv.shape[0] // seqlen, seqlen, nq, nkv, hd,
                             self.dropout_p if self.training else 0.0)
        r2 = residual.reshape(-1, residual.shape[-1]) if residual is not None else None
        y = tpar.row_output_linear(o, self.wo.weight, r2, self.tp,
                                   main_grad=main_grad_of(self.wo.weight), bias=self.wo.bias)
        return y.view(out_shape)
