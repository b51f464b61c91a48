"""DP-sharded sampler and loader (``src/data/dataloader.py:43-151``).

``ShardedSampler``: per-epoch permutation from ``Generator(seed + epoch)``
then the strided slice ``[rank::world]`` (disjoint, covering, sizes differ by
at most one).  TP peers share a dp rank and therefore see the same batches.
"""

from __future__ import annotations

from collections.abc import Iterator

import torch
from torch.utils.data import DataLoader, Dataset, Sampler


class ShardedSampler(Sampler[int]):
    def __init__(self, dataset_len: int, num_replicas: int, rank: int, shuffle: bool = True,
                 seed: int = 0) -> None:
        if not 0 <= rank < num_replicas:
            raise ValueError(f"rank={rank} out of range for num_replicas={num_replicas}.")
        self.dataset_len, self.num_replicas, self.rank = dataset_len, num_replicas, rank
        self.shuffle, self.seed, self.epoch = shuffle, seed, 0

    def set_epoch(self, epoch: int) -> None:
        self.epoch = epoch

    def __iter__(self) -> Iterator[int]:
        if self.shuffle:
            g = torch.Generator().manual_seed(self.seed + self.epoch)
            order = torch.randperm(self.dataset_len, generator=g).tolist()
        else:
            order = list(range(self.dataset_len))
        return iter(order[self.rank::self.num_replicas])

    def __len__(self) -> int:
        return len(range(self.rank, self.dataset_len, self.num_replicas))


def build_dataloader(dataset: Dataset, micro_batch_size: int, dp_size: int, dp_rank: int, *,
                     shuffle: bool = True, seed: int = 0, num_workers: int = 0,
                     drop_last: bool = True, pin_memory: bool = True) -> DataLoader:
    sampler = ShardedSampler(len(dataset), dp_size, dp_rank, shuffle, seed)  # type: ignore[arg-type]
    return DataLoader(dataset, batch_size=micro_batch_size, sampler=sampler,
                      num_workers=num_workers, drop_last=drop_last,
                      pin_memory=pin_memory and torch.cuda.is_available(),
                      persistent_workers=num_workers > 0)
