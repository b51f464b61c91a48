"""Autograd plumbing of the TP collectives and the parallel linear layers."""

import pytest
import torch
import torch.distributed as dist

from build_your_own_distributed_training_b200.parallel.tensor_parallel import (ColumnParallelLinear,
                                                                             RowParallelLinear,
                                                                             copy_to_tp_region,
                                                                             gather_from_tp_region,
                                                                             reduce_from_tp_region,
                                                                             scatter_to_tp_region)
from tests._dist_utils import run_distributed


@pytest.mark.parametrize("fn", [copy_to_tp_region, reduce_from_tp_region])
def test_fg_gradcheck_world1(single_process_pg, fn):
    x = torch.randn(3, 4, dtype=torch.float64, requires_grad=True)
    assert torch.autograd.gradcheck(lambda t: fn(t, dist.group.WORLD), (x,))


@pytest.mark.parametrize("fn", [gather_from_tp_region, scatter_to_tp_region])
def test_gather_scatter_gradcheck_world1(single_process_pg, fn):
    x = torch.randn(3, 4, dtype=torch.float64, requires_grad=True)
    assert torch.autograd.gradcheck(lambda t: fn(t, dist.group.WORLD, -1), (x,))


def test_tp1_equals_linear(single_process_pg):
    torch.manual_seed(0)
    col = ColumnParallelLinear(8, 6, dist.group.WORLD, bias=True)
    ref = torch.nn.Linear(8, 6)
    ref.weight.data.copy_(col.weight)
    ref.bias.data.copy_(col.bias)
    x = torch.randn(5, 8, requires_grad=True)
    xr = x.detach().clone().requires_grad_()
    col(x).sum().backward()
    ref(xr).sum().backward()
    assert torch.allclose(x.grad, xr.grad) and torch.allclose(col.weight.grad, ref.weight.grad)
    row = RowParallelLinear(8, 6, dist.group.WORLD, bias=False)
    assert torch.allclose(row(x), x @ row.weight.t())


def _divisibility(rank, world):
    with pytest.raises(ValueError, match="not divisible"):
        ColumnParallelLinear(4, 3, dist.group.WORLD)
    with pytest.raises(ValueError, match="not divisible"):
        RowParallelLinear(3, 4, dist.group.WORLD)


def test_divisibility_errors():
    run_distributed(_divisibility, 2)


def _column_row_chain(rank, world):
    torch.manual_seed(0)
    w1, w2 = torch.randn(8, 6), torch.randn(6, 8)
    x = torch.randn(4, 6, requires_grad=True)
    col = ColumnParallelLinear(6, 8, dist.group.WORLD, bias=False)
    row = RowParallelLinear(8, 6, dist.group.WORLD, bias=False)
    col.weight.data.copy_(w1.chunk(world, 0)[rank])
    row.weight.data.copy_(w2.chunk(world, 1)[rank])
    y = row(col(x))
    y.sum().backward()
    xr = x.detach().clone().requires_grad_()
    yr = (xr @ w1.t()) @ w2.t()
    yr.sum().backward()
    assert torch.allclose(y, yr, atol=1e-5)
    assert torch.allclose(x.grad, xr.grad, atol=1e-5)
    g = ColumnParallelLinear(6, 8, dist.group.WORLD, bias=False, gather_output=True)
    g.weight.data.copy_(w1.chunk(world, 0)[rank])
    assert torch.allclose(g(x), x @ w1.t(), atol=1e-5)


def test_column_row_chain_two_ranks():
    run_distributed(_column_row_chain, 2)
