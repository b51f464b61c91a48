"""Token embeddings (replicated and vocab-parallel) and the RoPE helpers.

Reference: ``src/model/embeddings.py:35-159``.  ``VocabParallelEmbedding``
is wired here: with ``parallel.loss_parallel`` the embedding and the LM head
are split over the TP group by vocabulary rows.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn as nn

from ..ops.embedding import embedding
from ..ops.rope import apply_rotary_emb, precompute_rope_cache  # noqa: F401
from .layers import main_grad_of


class TokenEmbedding(nn.Module):
    """Replicated ``[vocab, d_model]`` table, initialised ``N(0, 0.02)``."""

    def __init__(self, vocab_size: int, d_model: int) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.empty(vocab_size, d_model))
        nn.init.normal_(self.weight, mean=0.0, std=0.02)

    def forward(self, tokens: torch.Tensor, out_dtype: torch.dtype | None = None) -> torch.Tensor:
        return embedding(tokens, self.weight, main_grad=main_grad_of(self.weight), out_dtype=out_dtype)


class _SumOverTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):  # type: ignore[override]
        x = x.contiguous()
        dist.all_reduce(x, group=group)
        return x

    @staticmethod
    def backward(ctx, g):  # type: ignore[override]
        return g, None


class VocabParallelEmbedding(nn.Module):
    """Rows ``[rank * V/tp, (rank+1) * V/tp)`` live on TP rank ``rank``.

    Out-of-slice tokens look up row 0 and are zeroed; a TP all-reduce sums
    the partial lookups (reference ``src/model/embeddings.py:117-159``).
    """

    def __init__(self, vocab_size: int, d_model: int, tp_group: dist.ProcessGroup | None) -> None:
        super().__init__()
        self.tp_group = tp_group
        self.tp_size = dist.get_world_size(tp_group) if tp_group is not None else 1
        self.tp_rank = dist.get_rank(tp_group) if tp_group is not None else 0
        if vocab_size % self.tp_size:
            raise ValueError(f"vocab_size={vocab_size} is not divisible by tp_size={self.tp_size}.")
        self.vocab_per_partition = vocab_size // self.tp_size
        self.vocab_start = self.tp_rank * self.vocab_per_partition
        self.vocab_end = self.vocab_start + self.vocab_per_partition
        self.weight = nn.Parameter(torch.empty(self.vocab_per_partition, d_model))
        nn.init.normal_(self.weight, mean=0.0, std=0.02)

    def forward(self, tokens: torch.Tensor, out_dtype: torch.dtype | None = None,
                reduce: str = "all") -> torch.Tensor:
        """``reduce="all"``: all-reduce the partial lookups (every rank gets every
        token); ``"scatter"``: reduce-scatter them over the flattened tokens
        (sequence parallelism: each rank keeps its ``tokens/tp`` rows)."""
        outside = (tokens < self.vocab_start) | (tokens >= self.vocab_end)
        local = (tokens - self.vocab_start).masked_fill(outside, 0)
        out = embedding(local, self.weight, main_grad=main_grad_of(self.weight), out_dtype=out_dtype)
        out = out.masked_fill(outside.unsqueeze(-1), 0.0)
        if self.tp_size > 1:
            if reduce == "scatter":
                from ..parallel.tensor_parallel import reduce_scatter_rows_autograd
                return reduce_scatter_rows_autograd(out.reshape(-1, out.shape[-1]), self.tp_group)
            out = _SumOverTP.apply(out, self.tp_group)
        return out
