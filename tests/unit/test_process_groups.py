import pytest
import torch.distributed as dist

from build_your_own_distributed_training_b200.parallel.mesh import rank_coords, resolve_dp_size
from tests._dist_utils import run_distributed


def test_resolve_dp_size():
    assert resolve_dp_size(8, 2, -1) == 4
    assert resolve_dp_size(8, 8, -1) == 1
    with pytest.raises(ValueError, match="does not divide"):
        resolve_dp_size(8, 3, -1)
    with pytest.raises(ValueError, match="!= world_size"):
        resolve_dp_size(8, 2, 3)
    with pytest.raises(ValueError, match=">= 1"):
        resolve_dp_size(8, 0, -1)


def test_rank_coords_row_major():
    assert [rank_coords(r, 2) for r in range(4)] == [(0, 0), (0, 1), (1, 0), (1, 1)]


def _mesh_worker(rank, world, tp):
    from build_your_own_distributed_training_b200.parallel.process_groups import build_process_context
    ctx = build_process_context(tp_size=tp, backend="gloo", verbose=False)
    dp_rank, tp_rank = divmod(rank, tp)
    assert (ctx.dims.dp_rank, ctx.dims.tp_rank) == (dp_rank, tp_rank)
    assert ctx.dims.tp_size == tp and ctx.dims.dp_size == world // tp
    assert dist.get_world_size(ctx.tp_group) == tp
    assert dist.get_world_size(ctx.dp_group) == world // tp
    # tp group members are consecutive ranks
    assert dist.get_process_group_ranks(ctx.tp_group) == list(range(dp_rank * tp, dp_rank * tp + tp))
    ctx.barrier()


@pytest.mark.parametrize("tp", [1, 2, 4])
def test_mesh_layouts(tp):
    run_distributed(_mesh_worker, 4, tp)
