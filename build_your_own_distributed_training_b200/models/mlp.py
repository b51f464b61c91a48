"""SwiGLU feed-forward ``down(silu(gate(x)) * up(x))`` (reference ``src/model/mlp.py:40-72``).

``gate_proj`` and ``up_proj`` run as one GEMM on the stacked ``[W_gate; W_up]``
with the SwiGLU product computed in the epilogue; ``down_proj`` fuses the
residual add (and the TP reduction under tensor parallelism).
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..config import ModelConfig
from ..ops.linear import linear_swiglu
from ..parallel import tensor_parallel as tpar
from .layers import Linear, fused_rows, main_grad_of


class SwiGLUMLP(nn.Module):
    def __init__(self, config: ModelConfig) -> None:
        super().__init__()
        assert config.ffn_hidden_size is not None
        hidden = config.ffn_hidden_size
        self.gate_proj = Linear(config.d_model, hidden, config.mlp_bias)
        self.up_proj = Linear(config.d_model, hidden, config.mlp_bias)
        self.down_proj = Linear(hidden, config.d_model, config.mlp_bias)
        self.tp: tpar.TPInfo | None = None

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        out_shape = x.shape if residual is None else residual.shape
        x2, grad_comm = tpar.column_input_fused(x.reshape(-1, x.shape[-1]), self.tp,
                                                sp_ok=self.gate_proj.bias is None)
        ffn = self.gate_proj.weight.shape[0]
        if self.gate_proj.bias is not None:
            g = F.linear(x2, self.gate_proj.weight.to(x2.dtype), self.gate_proj.bias.to(x2.dtype))
            u = F.linear(x2, self.up_proj.weight.to(x2.dtype), self.up_proj.bias.to(x2.dtype))
            act = F.silu(g) * u
        else:
            w, mg = fused_rows([self.gate_proj.weight, self.up_proj.weight])
            act = linear_swiglu(x2, w, ffn, main_grad=mg, grad_comm=grad_comm)
        r2 = residual.reshape(-1, residual.shape[-1]) if residual is not None else None
        y = tpar.row_output_linear(act, self.down_proj.weight, r2, self.tp,
                                   main_grad=main_grad_of(self.down_proj.weight),
                                   bias=self.down_proj.bias)
        return y.view(out_shape)
