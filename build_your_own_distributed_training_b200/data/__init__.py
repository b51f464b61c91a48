"""Datasets, the dp-sharded sampler/loader and tokenizers."""

from .dataset import PackedTokenDataset, SyntheticTokenDataset, UniformTokenDataset  # noqa: F401
from .dataloader import ShardedSampler, build_dataloader  # noqa: F401
