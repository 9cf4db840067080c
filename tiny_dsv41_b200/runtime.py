"""Process/device bootstrap: one process per GPU, NCCL process group from the torchrun env.

API of ``dsv41_train/runtime.py:12-82`` (Runtime, initialize_runtime, local_tensor,
distributed_mean). CPU runs (tests) use gloo when WORLD_SIZE > 1.
"""

from __future__ import annotations

import datetime
import os
from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class Runtime:
    device: torch.device
    rank: int = 0
    local_rank: int = 0
    world_size: int = 1

    @property
    def distributed(self) -> bool:
        return self.world_size > 1

    @property
    def is_main(self) -> bool:
        return self.rank == 0


def choose_device(name: str) -> torch.device:
    if name == "auto":
        name = "cuda:0" if torch.cuda.is_available() else "cpu"
    return torch.device(name)


def initialize_runtime(
    device_name: str = "auto",
    local_rank_arg: int | None = None,
    *,
    require_distributed: bool = False,
    timeout_seconds: float | None = None,
) -> Runtime:
    """Bind the torchrun worker to its local GPU and create the process group.

    Single-process runs do not create a group unless ``require_distributed`` is set (a world of
    one still gets a group then, so collective code paths stay uniform).
    """
    world_size = int(os.environ.get("WORLD_SIZE", "1"))
    if world_size < 1:
        raise ValueError("WORLD_SIZE must be positive")
    if world_size == 1 and not require_distributed:
        return Runtime(device=choose_device(device_name))
    timeout = datetime.timedelta(seconds=timeout_seconds) if timeout_seconds else None
    use_cuda = torch.cuda.is_available() and device_name in {"auto", "cuda"}
    if not use_cuda:
        if not dist.is_initialized():
            os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
            os.environ.setdefault("MASTER_PORT", "29512")
            os.environ.setdefault("RANK", "0")
            os.environ.setdefault("WORLD_SIZE", "1")
            kwargs = {"backend": "gloo"}
            if timeout:
                kwargs["timeout"] = timeout
            dist.init_process_group(**kwargs)
        return Runtime(torch.device("cpu"), dist.get_rank(), int(os.environ.get("LOCAL_RANK", "0")),
                       dist.get_world_size())
    local_rank_value = os.environ.get("LOCAL_RANK")
    local_rank = int(local_rank_value) if local_rank_value is not None else (local_rank_arg or 0)
    if not 0 <= local_rank < torch.cuda.device_count():
        raise RuntimeError(f"LOCAL_RANK {local_rank} is outside the {torch.cuda.device_count()} visible devices")
    torch.cuda.set_device(local_rank)
    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29512")
        os.environ.setdefault("RANK", "0")
        os.environ.setdefault("WORLD_SIZE", "1")
        kwargs = {"backend": "nccl", "device_id": torch.device("cuda", local_rank)}
        if timeout:
            kwargs["timeout"] = timeout
        dist.init_process_group(**kwargs)
    return Runtime(torch.device("cuda", local_rank), dist.get_rank(), local_rank, dist.get_world_size())


def local_tensor(tensor: torch.Tensor) -> torch.Tensor:
    return tensor.to_local() if hasattr(tensor, "to_local") else tensor


def distributed_mean(value: torch.Tensor, runtime: Runtime) -> float:
    value = value.detach().float()
    if runtime.distributed and dist.is_initialized():
        value = value.clone()
        dist.all_reduce(value, op=dist.ReduceOp.SUM)
        value /= runtime.world_size
    return value.item()


__all__ = ["Runtime", "choose_device", "distributed_mean", "initialize_runtime", "local_tensor"]
