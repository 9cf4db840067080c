"""Query-LoRA profile shared by the learner and the rollout service
(``dsv41_train/rl/lora_config.py:28-79``: same fields, ranks and JSON form).

Adapters sit on the query down-projection (``attention.q_a``; vLLM name ``attn.wq_a``) of the
selected layers (``None`` = all), dropout is zero so scored probabilities are exact, and the rank
is one the service's kernels support.
"""

from __future__ import annotations

import math
import re
from collections.abc import Mapping
from dataclasses import dataclass

SUPPORTED_LORA_RANKS = (8, 16, 32, 64, 128)


def parse_lora_layers(value: str) -> tuple[int, ...] | None:
    if not isinstance(value, str):
        raise ValueError("LoRA layers must be 'all' or comma-separated layer indices")
    if value.strip() == "all":
        return None
    parts = [p.strip() for p in value.split(",")]
    if not parts or any(re.fullmatch(r"[0-9]+", p) is None for p in parts):
        raise ValueError("LoRA layers must be 'all' or comma-separated nonnegative indices")
    layers = tuple(int(p) for p in parts)
    if len(set(layers)) != len(layers):
        raise ValueError("LoRA layer indices must be distinct")
    return tuple(sorted(layers))


@dataclass(frozen=True)
class DistributedLoRAConfig:
    rank: int = 8
    alpha: float = 8.0
    layers: tuple[int, ...] | None = None

    def __post_init__(self):
        if type(self.rank) is not int or self.rank not in SUPPORTED_LORA_RANKS:
            raise ValueError(f"LoRA rank must be one of {SUPPORTED_LORA_RANKS}")
        if type(self.alpha) not in (int, float) or not math.isfinite(self.alpha) or self.alpha <= 0:
            raise ValueError("LoRA alpha must be finite and positive")
        if self.layers is not None:
            if (not isinstance(self.layers, tuple) or not self.layers
                    or any(type(x) is not int or x < 0 for x in self.layers) or len(set(self.layers)) != len(self.layers)):
                raise ValueError("LoRA layers must be distinct nonnegative indices or None")
            object.__setattr__(self, "layers", tuple(sorted(self.layers)))
        object.__setattr__(self, "alpha", float(self.alpha))

    def selected_layers(self, num_layers: int) -> tuple[int, ...]:
        if type(num_layers) is not int or num_layers < 1:
            raise ValueError("backbone layer count must be a positive integer")
        layers = tuple(range(num_layers)) if self.layers is None else self.layers
        if layers[-1] >= num_layers:
            raise ValueError(f"LoRA layer index is outside the {num_layers}-layer backbone")
        return layers

    def parameter_count(self, hidden: int, q_rank: int, num_layers: int) -> int:
        if any(type(n) is not int or n < 1 for n in (hidden, q_rank)):
            raise ValueError("query projection dimensions must be positive integers")
        return len(self.selected_layers(num_layers)) * self.rank * (hidden + q_rank)

    def to_dict(self) -> dict:
        return {"rank": self.rank, "alpha": self.alpha, "layers": list(self.layers) if self.layers is not None else None}

    @classmethod
    def from_dict(cls, value: Mapping) -> "DistributedLoRAConfig":
        if not isinstance(value, Mapping) or set(value) != {"rank", "alpha", "layers"}:
            raise ValueError("LoRA configuration requires exactly rank, alpha and layers")
        layers = value["layers"]
        if layers is not None and not isinstance(layers, list):
            raise ValueError("serialized LoRA layers must be a list or null")
        return cls(rank=value["rank"], alpha=value["alpha"], layers=tuple(layers) if layers is not None else None)

    def lora_config(self):
        """The learner-side ``LoRAConfig`` (query down-projection only, no dropout)."""
        from ..lora import LoRAConfig

        return LoRAConfig(self.rank, self.alpha, 0.0, ("attention.q_a",))


__all__ = ["DistributedLoRAConfig", "SUPPORTED_LORA_RANKS", "parse_lora_layers"]
