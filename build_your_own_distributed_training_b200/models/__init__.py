"""LLaMA-style decoder with the reference's module and parameter names."""

from .transformer import RMSNorm, Transformer, TransformerBlock, build_model  # noqa: F401
from .attention import Attention  # noqa: F401
from .mlp import SwiGLUMLP  # noqa: F401
from .embeddings import TokenEmbedding, VocabParallelEmbedding  # noqa: F401
