"""Device meshes for dense (FSDP x CP) and sparse (expert-FSDP x EP) parameters.

Same mesh names as ``dsv41_train/parallel.py:15-73``. Unlike the reference drivers, CP and EP
are independent dimensions (e.g. CP2 x EP4 on 8 GPUs).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import TYPE_CHECKING

import torch.distributed as dist

if TYPE_CHECKING:
    from torch.distributed.device_mesh import DeviceMesh


@dataclass(frozen=True)
class ParallelMeshes:
    fsdp: "DeviceMesh | None"
    cp: "DeviceMesh | None"
    ep: "DeviceMesh | None"
    expert_fsdp: "DeviceMesh | None"
    dense: "DeviceMesh | None" = None
    sparse: "DeviceMesh | None" = None
    engram: "DeviceMesh | None" = None
    world: "DeviceMesh | None" = None

    @property
    def dense_world(self) -> "DeviceMesh | None":
        """1-D mesh over every rank (dense FSDP when context parallelism splits sequences)."""
        return self.world

    @property
    def cp_size(self) -> int:
        return 1 if self.cp is None else self.cp.size()

    @property
    def ep_size(self) -> int:
        return 1 if self.ep is None else self.ep.size()

    @classmethod
    def build(cls, *, cp: int = 1, ep: int = 1, device_type: str = "cuda", engram: bool = False) -> "ParallelMeshes":
        from torch.distributed.device_mesh import init_device_mesh

        if not dist.is_initialized():
            raise RuntimeError("initialize torch.distributed before building parallel meshes")
        world = dist.get_world_size()
        if cp < 1 or world % cp:
            raise ValueError(f"cp ({cp}) must divide world size ({world})")
        if ep < 1 or world % ep:
            raise ValueError(f"ep ({ep}) must divide world size ({world})")
        dense = init_device_mesh(device_type, (world // cp, cp), mesh_dim_names=("fsdp", "cp"))
        sparse = init_device_mesh(device_type, (world // ep, ep), mesh_dim_names=("expert_fsdp", "ep"))
        world_mesh = init_device_mesh(device_type, (world,), mesh_dim_names=("world",))
        engram_mesh = world_mesh if engram else None
        return cls(
            fsdp=dense["fsdp"],
            cp=dense["cp"] if cp > 1 else None,
            ep=sparse["ep"] if ep > 1 else None,
            expert_fsdp=sparse["expert_fsdp"],
            dense=dense,
            sparse=sparse,
            engram=engram_mesh,
            world=world_mesh,
        )


__all__ = ["ParallelMeshes"]
