import torch

from build_your_own_distributed_training_b200.data.dataloader import ShardedSampler, build_dataloader
from build_your_own_distributed_training_b200.data.dataset import (PackedTokenDataset, SyntheticTokenDataset,
                                                                   UniformTokenDataset, write_uniform_token_file)


def test_partition_exact_and_disjoint():
    parts = [list(ShardedSampler(103, 4, r, shuffle=True, seed=5)) for r in range(4)]
    flat = sum(parts, [])
    assert sorted(flat) == list(range(103))
    assert max(map(len, parts)) - min(map(len, parts)) <= 1


def test_epoch_reshuffles():
    s = ShardedSampler(50, 2, 0, shuffle=True, seed=1)
    a = list(s)
    s.set_epoch(1)
    assert list(s) != a


def test_datasets(tmp_path):
    d = SyntheticTokenDataset(64, 16, 10, seed=3)
    x = d[2]
    assert torch.equal(x["input_ids"][1:], x["labels"][:-1])
    assert torch.equal(d[2]["input_ids"], x["input_ids"])
    u = UniformTokenDataset(1000, 32, 5, seed=0)
    assert u[1]["input_ids"].max() < 1000 and torch.equal(u[1]["labels"], UniformTokenDataset(1000, 32, 5, 0)[1]["labels"])
    path = write_uniform_token_file(str(tmp_path / "t.bin"), 500, 1000)
    p = PackedTokenDataset(path, 32)
    assert len(p) == (1000 - 1) // 32 and p[0]["input_ids"].shape == (32,)
    dl = build_dataloader(u, 2, 1, 0, shuffle=False)
    assert next(iter(dl))["input_ids"].shape == (2, 32)
