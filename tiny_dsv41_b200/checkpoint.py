"""Distributed (DCP) training checkpoints for the generic training entry points.

Same contract as ``dsv41_train/checkpoint.py``: a ``TrainingState`` (model, optimizer, model
config, per-rank data generator state, step) saved with ``torch.distributed.checkpoint`` under
``<folder>/step-<N>``; a directory counts only once its ``.metadata`` file exists; loading
checks the model config and world size (the data generators are per rank). DCP shards and
reshards the model and optimizer states itself, so sharded (FSDP2) and single-device models
use the same code.
"""

from __future__ import annotations

import re
from pathlib import Path
from typing import Any

import torch
import torch.distributed as dist
import torch.distributed.checkpoint as dcp
from torch import nn
from torch.distributed.checkpoint.state_dict import StateDictOptions, get_state_dict, set_state_dict
from torch.distributed.checkpoint.stateful import Stateful


def _position() -> tuple[int, int]:
    return (dist.get_rank(), dist.get_world_size()) if dist.is_initialized() else (0, 1)


class TrainingState(Stateful):
    def __init__(self, model: nn.Module, optimizer: torch.optim.Optimizer, *, model_config: dict[str, Any],
                 data_generator: torch.Generator) -> None:
        self.model = model
        self.optimizer = optimizer
        self.model_config = model_config
        self.data_generator = data_generator
        self.step = 0

    def state_dict(self) -> dict[str, Any]:
        model_state, optim_state = get_state_dict(self.model, self.optimizer)
        rank, world = _position()
        return {"model": model_state, "optimizer": optim_state, "model_config": self.model_config,
                "data_generator": {"world_size": world, f"rank-{rank}": self.data_generator.get_state()},
                "step": self.step}

    def load_state_dict(self, state: dict[str, Any]) -> None:
        if state["model_config"] != self.model_config:
            raise ValueError("checkpoint model config does not match the current model")
        rank, world = _position()
        generators = state["data_generator"]
        if generators["world_size"] != world:
            raise ValueError("cannot restore the data generator after changing world size")
        # parameters that never received a gradient have no optimizer state (strict=False)
        set_state_dict(self.model, self.optimizer, model_state_dict=state["model"],
                       optim_state_dict=state["optimizer"], options=StateDictOptions(strict=False))
        self.data_generator.set_state(generators[f"rank-{rank}"])
        self.step = int(state["step"])


class CheckpointManager:
    _STEP = re.compile(r"step-(0|[1-9]\d*)")

    def __init__(self, folder, state: TrainingState) -> None:
        self.folder = Path(folder)
        self.state = state

    def _path(self, step: int) -> Path:
        return self.folder / f"step-{step}"

    @torch.no_grad()
    def save(self, step: int) -> Path:
        if step < 0:
            raise ValueError("checkpoint step must be non-negative")
        self.state.step = step
        path = self._path(step)
        dcp.save({"train": self.state}, checkpoint_id=str(path))
        return path

    @torch.no_grad()
    def load(self, step: int | None = None) -> int:
        step = self.latest_step() if step is None else step
        if step is None:
            raise FileNotFoundError(f"no checkpoint found in {self.folder}")
        if step < 0:
            raise ValueError("checkpoint step must be non-negative")
        path = self._path(step)
        if not (path / ".metadata").is_file():
            raise FileNotFoundError(f"checkpoint is incomplete or missing: {path}")
        self._prime_optimizer(path)
        dcp.load({"train": self.state}, checkpoint_id=str(path))
        return self.state.step

    def _prime_optimizer(self, path: Path) -> None:
        """Create optimizer state for exactly the parameters that have state in the checkpoint.

        Parameters that never received a gradient (e.g. sparse indexers trained by no loss) have
        no optimizer state when saved; a fresh optimizer would otherwise be initialised for every
        parameter and ask the checkpoint for keys it does not hold. The throw-away step below is
        overwritten by the load."""
        prefix = "train.optimizer.state."
        keys = dcp.FileSystemReader(str(path)).read_metadata().state_dict_metadata.keys()
        names = {k[len(prefix):].rsplit(".", 1)[0] for k in keys if k.startswith(prefix)}
        model, optimizer = self.state.model, self.state.optimizer
        params = [p for n, p in model.named_parameters() if n in names and p not in optimizer.state]
        if not params:
            return
        for p in params:
            p.grad = torch.zeros_like(p)
        optimizer.step()
        optimizer.zero_grad(set_to_none=True)

    def latest_step(self) -> int | None:
        if not self.folder.is_dir():
            return None
        steps = [int(m.group(1)) for p in self.folder.iterdir()
                 if (m := self._STEP.fullmatch(p.name)) is not None and (p / ".metadata").is_file()]
        return max(steps, default=None)


__all__ = ["CheckpointManager", "TrainingState"]
