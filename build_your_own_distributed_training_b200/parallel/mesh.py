"""The named ``(dp, tp)`` device mesh.

Global rank ``r`` sits at ``(dp_rank, tp_rank) = divmod(r, tp_size)``: the
ranks of one tensor-parallel group are consecutive, so on one 8-GPU box a TP
pair is two neighbouring GPUs and every TP collective stays inside the
NVSwitch domain.  The mesh is always 2-D; a size-1 axis is a valid degenerate
group (reference ``src/parallelism/mesh.py:10-233``).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import cast

import torch
import torch.distributed as dist
from torch.distributed.device_mesh import DeviceMesh, init_device_mesh


@dataclass(frozen=True)
class ParallelDims:
    tp_size: int
    dp_size: int
    world_size: int
    dp_rank: int
    tp_rank: int
    global_rank: int

    @property
    def tp_enabled(self) -> bool:
        return self.tp_size > 1

    @property
    def dp_enabled(self) -> bool:
        return self.dp_size > 1


def resolve_dp_size(world_size: int, tp_size: int, dp_size: int) -> int:
    """Infer ``dp`` from ``world // tp`` when ``dp_size == -1``; check the product."""
    if tp_size < 1:
        raise ValueError(f"tp_size must be >= 1, got {tp_size}.")
    if world_size % tp_size:
        ok = [t for t in range(1, world_size + 1) if world_size % t == 0]
        raise ValueError(
            f"tp_size={tp_size} does not divide world_size={world_size}; pick one of {ok}."
        )
    dp = world_size // tp_size if dp_size == -1 else dp_size
    if dp * tp_size != world_size:
        raise ValueError(
            f"dp_size({dp}) x tp_size({tp_size}) = {dp * tp_size} != world_size({world_size})."
        )
    return dp


def rank_coords(global_rank: int, tp_size: int) -> tuple[int, int]:
    """``(dp_rank, tp_rank)`` of a global rank in the row-major layout."""
    return divmod(global_rank, tp_size)


def build_device_mesh(tp_size: int, dp_size: int = -1, device_type: str | None = None) -> DeviceMesh:
    if not dist.is_initialized():
        raise RuntimeError("build_device_mesh needs an initialised default process group.")
    dp = resolve_dp_size(dist.get_world_size(), tp_size, dp_size)
    if device_type is None:
        device_type = "cuda" if torch.cuda.is_available() else "cpu"
    return init_device_mesh(device_type, (dp, tp_size), mesh_dim_names=("dp", "tp"))


def get_parallel_dims(mesh: DeviceMesh) -> ParallelDims:
    tp, dp = mesh["tp"].size(), mesh["dp"].size()
    return ParallelDims(tp, dp, tp * dp, mesh["dp"].get_local_rank(),
                        mesh["tp"].get_local_rank(), dist.get_rank())


def get_dp_group(mesh: DeviceMesh) -> dist.ProcessGroup:
    return cast(dist.ProcessGroup, mesh["dp"].get_group())


def get_tp_group(mesh: DeviceMesh) -> dist.ProcessGroup:
    return cast(dist.ProcessGroup, mesh["tp"].get_group())


def format_mesh_layout(mesh: DeviceMesh) -> str:
    """Human-readable table of global ranks by (dp, tp) coordinate."""
    grid = mesh.mesh
    dp, tp = grid.shape
    lines = [f"DeviceMesh layout (dp_size={dp}, tp_size={tp}):",
             "        " + "".join(f"tp={t:<6}" for t in range(tp))]
    for d in range(dp):
        lines.append(f"  dp={d:<3} " + "".join(f"r{int(grid[d, t]):<6}" for t in range(tp)))
    return "\n".join(lines)
