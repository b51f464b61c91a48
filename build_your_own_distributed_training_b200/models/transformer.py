"""The decoder: embedding -> N pre-norm blocks -> RMSNorm -> LM head.

Structure, initialisation and parameter names follow
``src/model/transformer.py:47-197``: ``N(0, 0.02)`` for the embedding and all
projections, ``N(0, 0.02/sqrt(2L))`` for ``wo``/``down_proj``, ones for norms,
optional tied head, non-persistent RoPE buffers.  ``TransformerBlock`` is the
sharding/recompute unit.  Differences:

* the residual add is fused into the output projections;
* with labels the loss comes from the fused head+cross-entropy op; set
  ``return_logits = False`` to skip keeping the ``[tokens, vocab]`` logits
  (the trainer does);
* under sequence parallelism the residual stream between blocks holds only
  this TP rank's tokens, and the head + loss run on those tokens only (the
  loss is then combined over the TP group), so no rank repeats head work.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from ..config import ModelConfig
from ..ops.loss import lm_head_cross_entropy
from ..ops.norm import rms_norm
from ..ops.rope import precompute_rope_cache
from ..parallel import tensor_parallel as tpar
from .attention import Attention
from .embeddings import TokenEmbedding, VocabParallelEmbedding
from .layers import Linear, main_grad_of
from .mlp import SwiGLUMLP


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float = 1e-5) -> None:
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return rms_norm(x, self.weight, self.eps, main_grad=main_grad_of(self.weight))


class TransformerBlock(nn.Module):
    def __init__(self, config: ModelConfig, layer_id: int) -> None:
        super().__init__()
        self.layer_id = layer_id
        self.attention_norm = RMSNorm(config.d_model, config.norm_eps)
        self.attention = Attention(config)
        self.mlp_norm = RMSNorm(config.d_model, config.norm_eps)
        self.mlp = SwiGLUMLP(config)

    def forward(self, x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        h = self.attention(self.attention_norm(x), cos, sin, residual=x)
        return self.mlp(self.mlp_norm(h), residual=h)


class Transformer(nn.Module):
    def __init__(self, config: ModelConfig) -> None:
        super().__init__()
        self.config = config
        self.tok_embeddings: nn.Module = TokenEmbedding(config.vocab_size, config.d_model)
        self.layers = nn.ModuleList(TransformerBlock(config, i) for i in range(config.n_layers))
        self.norm = RMSNorm(config.d_model, config.norm_eps)
        self.lm_head = Linear(config.d_model, config.vocab_size, bias=False)
        if config.tie_embeddings:
            self.lm_head.weight = self.tok_embeddings.weight
        cos, sin = precompute_rope_cache(config.head_dim, config.max_seq_len, config.rope_theta)
        self.register_buffer("rope_cos", cos, persistent=False)
        self.register_buffer("rope_sin", sin, persistent=False)
        self.return_logits = True
        self.tp: tpar.TPInfo | None = None
        self._init_weights()

    def _init_weights(self) -> None:
        for m in self.modules():
            if isinstance(m, Linear):
                nn.init.normal_(m.weight, mean=0.0, std=0.02)
                if m.bias is not None:
                    nn.init.zeros_(m.bias)
        std = 0.02 / (2 * self.config.n_layers) ** 0.5
        for blk in self.layers:
            nn.init.normal_(blk.attention.wo.weight, mean=0.0, std=std)
            nn.init.normal_(blk.mlp.down_proj.weight, mean=0.0, std=std)

    def embed(self, tokens: torch.Tensor) -> torch.Tensor:
        if not tpar.sp_on(self.tp):
            return self.tok_embeddings(tokens)
        if isinstance(self.tok_embeddings, VocabParallelEmbedding):
            # partial lookups of every token, summed and split by tokens in one reduce-scatter
            return self.tok_embeddings(tokens.reshape(-1), reduce="scatter")
        # replicated table: look up only this rank's tokens; its gradient is partial
        # and the sharding engine sums replicated gradients over the TP group
        return self.tok_embeddings(tpar.sequence_slice(tokens.reshape(-1), self.tp))

    def head(self, h: torch.Tensor, labels: torch.Tensor | None
             ) -> tuple[torch.Tensor | None, torch.Tensor | None]:
        h = self.norm(h)
        h2 = h.reshape(-1, h.shape[-1])
        w = self.lm_head.weight
        mg = main_grad_of(w)
        if isinstance(self.tok_embeddings, VocabParallelEmbedding):
            return tpar.vocab_parallel_head_ce(h2, w, labels, self.tp, main_grad=mg,
                                               vocab_start=self.tok_embeddings.vocab_start)
        if tpar.sp_on(self.tp):
            lab = None if labels is None else tpar.sequence_slice(labels.reshape(-1), self.tp)
            return tpar.sequence_parallel_head_ce(h2, w, lab, self.tp, main_grad=mg)
        logits, loss = lm_head_cross_entropy(h2, w, None if labels is None else labels.reshape(-1),
                                             main_grad=mg, return_logits=self.return_logits
                                             or labels is None)
        return logits, loss

    def forward(self, tokens: torch.Tensor, labels: torch.Tensor | None = None
                ) -> tuple[torch.Tensor | None, torch.Tensor | None]:
        """``tokens``/``labels``: ``[batch, seq]``; returns ``(logits, loss)``.

        ``logits`` is ``[batch, seq, vocab]`` (``None`` when ``return_logits``
        is off, or under sequence/loss parallelism).
        """
        bsz, seqlen = tokens.shape
        cos, sin = self.rope_cos[:seqlen], self.rope_sin[:seqlen]
        h = self.embed(tokens)
        for layer in self.layers:
            h = layer(h, cos, sin)
        logits, loss = self.head(h, labels)
        if logits is not None and logits.dim() == 2 and logits.shape[0] == bsz * seqlen:
            logits = logits.view(bsz, seqlen, -1)
        return logits, loss


def build_model(config: ModelConfig) -> Transformer:
    return Transformer(config)
