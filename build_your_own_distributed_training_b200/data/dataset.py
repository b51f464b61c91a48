"""Token datasets yielding ``{"input_ids": [S], "labels": [S]}`` (labels shifted by one).

* ``SyntheticTokenDataset``: a learnable Markov corpus (a fixed random table of
  ``k`` successors per token; same construction as
  ``src/data/dataset.py:39-90``, sampled with vectorised draws, so its token
  stream is not bit-identical to the reference's).
* ``UniformTokenDataset``: uniform-random ids in ``[0, vocab)``; sample ``i``
  is a pure function of ``(seed, i)``.  This is the synthetic workload of the
  throughput benchmarks.
* ``PackedTokenDataset``: a flat uint16 token file read through ``np.memmap``
  in non-overlapping windows of ``seq_len + 1`` (``src/data/dataset.py:93-138``).
"""

from __future__ import annotations

import os

import numpy as np
import torch
from torch.utils.data import Dataset


def _pair(seq: torch.Tensor) -> dict[str, torch.Tensor]:
    return {"input_ids": seq[:-1].contiguous(), "labels": seq[1:].contiguous()}


class SyntheticTokenDataset(Dataset):
    def __init__(self, vocab_size: int, seq_len: int, num_samples: int, seed: int = 0,
                 k: int = 4) -> None:
        self.vocab_size, self.seq_len, self.num_samples, self.seed = vocab_size, seq_len, num_samples, seed
        self.k = min(k, vocab_size)
        g = torch.Generator().manual_seed(seed)
        self.next_tokens = torch.randint(0, vocab_size, (vocab_size, self.k), generator=g)
        self._table = self.next_tokens.numpy()

    def __len__(self) -> int:
        return self.num_samples

    def __getitem__(self, idx: int) -> dict[str, torch.Tensor]:
        g = torch.Generator().manual_seed(self.seed * 1_000_003 + idx)
        first = int(torch.randint(0, self.vocab_size, (1,), generator=g))
        choice = torch.randint(0, self.k, (self.seq_len,), generator=g).numpy()
        seq = np.empty(self.seq_len + 1, dtype=np.int64)
        seq[0] = first
        tab = self._table
        for t in range(1, self.seq_len + 1):
            seq[t] = tab[seq[t - 1], choice[t - 1]]
        return _pair(torch.from_numpy(seq))


class UniformTokenDataset(Dataset):
    def __init__(self, vocab_size: int, seq_len: int, num_samples: int, seed: int = 0) -> None:
        self.vocab_size, self.seq_len, self.num_samples, self.seed = vocab_size, seq_len, num_samples, seed

    def __len__(self) -> int:
        return self.num_samples

    def __getitem__(self, idx: int) -> dict[str, torch.Tensor]:
        g = torch.Generator().manual_seed(self.seed * 1_000_003 + idx)
        return _pair(torch.randint(0, self.vocab_size, (self.seq_len + 1,), generator=g))


class PackedTokenDataset(Dataset):
    def __init__(self, path: str, seq_len: int) -> None:
        if not os.path.exists(path):
            raise FileNotFoundError(f"Token corpus not found: {path}")
        self.path, self.seq_len = path, seq_len
        self._data: np.memmap | None = None
        n = os.path.getsize(path) // np.dtype(np.uint16).itemsize
        if n < seq_len + 1:
            raise ValueError(f"Corpus has {n} tokens < seq_len+1={seq_len + 1}.")
        self.num_windows = (n - 1) // seq_len

    def _mm(self) -> np.memmap:
        if self._data is None:  # opened lazily so each loader worker maps its own copy
            self._data = np.memmap(self.path, dtype=np.uint16, mode="r")
        return self._data

    def __len__(self) -> int:
        return self.num_windows

    def __getitem__(self, idx: int) -> dict[str, torch.Tensor]:
        s = idx * self.seq_len
        chunk = np.asarray(self._mm()[s:s + self.seq_len + 1], dtype=np.int64)
        return _pair(torch.from_numpy(chunk))


def write_uniform_token_file(path: str, vocab_size: int, n_tokens: int, seed: int = 0) -> str:
    """Write ``n_tokens`` uniform-random uint16 ids (for packed-file workloads)."""
    if vocab_size > 65536:
        raise ValueError("uint16 token files hold vocab sizes up to 65536")
    rng = np.random.default_rng(seed)
    rng.integers(0, vocab_size, size=n_tokens, dtype=np.uint16).tofile(path)
    return path
