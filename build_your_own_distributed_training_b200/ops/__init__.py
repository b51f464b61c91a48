"""Fused operators.

Every op has two paths chosen by the device of its inputs:

* CUDA: this package's sm_100a kernels from the ``_C`` extension (tcgen05/TMEM
  GEMMs with fused epilogues, fused RMSNorm, attention, cross-entropy, AdamW).
* CPU: plain PyTorch restating the reference's math in fp32; it backs the
  gloo tests and is the numerical oracle of the kernel tests.
"""

from .linear import linear, linear_qkv_rope, linear_swiglu  # noqa: F401
from .norm import rms_norm  # noqa: F401
from .rope import apply_rotary_emb, precompute_rope_cache  # noqa: F401
from .attention import causal_attention  # noqa: F401
from .loss import lm_head_cross_entropy  # noqa: F401
from .embedding import embedding  # noqa: F401
