"""ParallelContext: rank -> (dp_rank, tp_rank) on a 2-D ``("dp", "tp")`` DeviceMesh.

Same mapping as the reference (mint/utils/parallel.py:15-87): consecutive ranks share a TP
group (``dp_rank = rank // tp``, ``tp_rank = rank % tp``); the dp group is WORLD when tp == 1.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Any

import torch.distributed as dist
from torch.distributed.device_mesh import DeviceMesh, init_device_mesh


def dp_tp_ranks(rank: int, tp_size: int) -> tuple[int, int]:
    return rank // tp_size, rank % tp_size


@dataclass(frozen=True)
class ParallelContext:
    rank: int = 0
    world_size: int = 1
    dp_rank: int = 0
    dp_size: int = 1
    tp_rank: int = 0
    tp_size: int = 1
    ddp_level: int = 0
    sp: bool = False
    dp_group: Any = None
    tp_group: Any = None
    mesh: DeviceMesh | None = None

    @classmethod
    def build(
        cls,
        *,
        tp_size: int = 1,
        ddp_level: int = 0,
        sp: bool = False,
        device_type: str = "cpu",
    ) -> ParallelContext:
        if ddp_level not in (0, 1, 2, 3):
            raise ValueError(f"ddp_level must be 0..3, got {ddp_level}")
        if not (dist.is_available() and dist.is_initialized()):
            if tp_size != 1:
                raise ValueError(f"tp_size={tp_size} requires a distributed launch")
            return cls(rank=int(os.getenv("RANK", "0")), world_size=int(os.getenv("WORLD_SIZE", "1")),
                       ddp_level=ddp_level, sp=sp)
        rank, world = dist.get_rank(), dist.get_world_size()
        if tp_size < 1 or world % tp_size != 0:
            raise ValueError(f"world_size={world} is not divisible by tp_size={tp_size}")
        if tp_size == 1:
            return cls(rank=rank, world_size=world, dp_rank=rank, dp_size=world, ddp_level=ddp_level,
                       sp=sp, dp_group=dist.group.WORLD)
        dp_size = world // tp_size
        mesh = init_device_mesh(device_type, (dp_size, tp_size), mesh_dim_names=("dp", "tp"))
        dp_rank, tp_rank = dp_tp_ranks(rank, tp_size)
        return cls(rank=rank, world_size=world, dp_rank=dp_rank, dp_size=dp_size, tp_rank=tp_rank,
                   tp_size=tp_size, ddp_level=ddp_level, sp=sp, dp_group=mesh.get_group("dp"),
                   tp_group=mesh.get_group("tp"), mesh=mesh)

    @property
    def is_main(self) -> bool:
        return self.rank == 0
