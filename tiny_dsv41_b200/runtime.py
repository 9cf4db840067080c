"""Process and device bootstrap: one process per GPU, the NCCL process group from the torchrun
environment (gloo for CPU runs with WORLD_SIZE > 1, as the multi-rank tests use).

Public names follow ``dsv41_train/runtime.py:12-82`` (``Runtime``, ``initialize_runtime``,
``local_tensor``, ``distributed_mean``) so entry points written against either load the same way.
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


def _env_defaults() -> None:
    """A single process started without torchrun still gets a (world of one) process group."""
    for key, value in (("MASTER_ADDR", "127.0.0.1"), ("MASTER_PORT", "29512"), ("RANK", "0"), ("WORLD_SIZE", "1")):
        os.environ.setdefault(key, value)


def _open_group(backend: str, timeout: datetime.timedelta | None, device: torch.device | None) -> None:
    if dist.is_initialized():
        return
    _env_defaults()
    options = {"backend": backend}
    if timeout is not None:
        options["timeout"] = timeout
    if device is not None:
        options["device_id"] = device
    dist.init_process_group(**options)


def initialize_runtime(
    device_name: str = "auto",
    local_rank_arg: int | None = None,
    *,
    require_distributed: bool = False,
    timeout_seconds: float | None = None,
) -> Runtime:
    """Bind this torchrun worker to its local GPU and open the process group (NCCL on GPUs, gloo
    on CPU runs). A single process opens no group unless ``require_distributed`` is set; then it
    opens a world of one, so collective code paths stay the same."""
    world_size = int(os.environ.get("WORLD_SIZE", "1"))
    if world_size < 1:
        raise ValueError("WORLD_SIZE must be positive")
    if world_size == 1 and not require_distributed:
        return Runtime(device=choose_device(device_name))
    timeout = datetime.timedelta(seconds=timeout_seconds) if timeout_seconds else None
    if not (torch.cuda.is_available() and device_name in ("auto", "cuda")):
        _open_group("gloo", timeout, None)
        return Runtime(torch.device("cpu"), dist.get_rank(), int(os.environ.get("LOCAL_RANK", "0")),
                       dist.get_world_size())
    env_rank = os.environ.get("LOCAL_RANK")
    local_rank = int(env_rank) if env_rank is not None else (local_rank_arg or 0)
    if not 0 <= local_rank < torch.cuda.device_count():
        raise RuntimeError(f"LOCAL_RANK {local_rank} is outside the {torch.cuda.device_count()} visible devices")
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    _open_group("nccl", timeout, device)
    return Runtime(device, dist.get_rank(), local_rank, dist.get_world_size())


def local_tensor(tensor: torch.Tensor) -> torch.Tensor:
    return tensor.to_local() if hasattr(tensor, "to_local") else tensor


def distributed_mean(value: torch.Tensor, runtime: Runtime) -> float:
    """Mean of a scalar over all ranks (the value itself on a single process)."""
    total = value.detach().float().clone()
    if runtime.distributed and dist.is_initialized():
        dist.all_reduce(total, op=dist.ReduceOp.SUM)
        return total.item() / runtime.world_size
    return total.item()


__all__ = ["Runtime", "choose_device", "distributed_mean", "initialize_runtime", "local_tensor"]
