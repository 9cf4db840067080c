"""Parallel runtime: meshes, context parallelism, expert-parallel dispatch, FSDP glue."""

from .cp import ContextParallel, ModelContext, pack_sequences
from .meshes import ParallelMeshes

__all__ = ["ContextParallel", "ModelContext", "ParallelMeshes", "pack_sequences"]
