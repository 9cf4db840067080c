"""Query-LoRA profile shared by the distributed learner and the rollout service.

Same fields, supported ranks and JSON form as ``dsv41_train/rl/lora_config.py:28-79`` (the service
validates the profile it receives). Adapters sit on the query down-projection of the selected
decoder layers (``attention.q_a`` here, ``attn.wq_a`` in the service), with zero dropout so the
probabilities the learner scores are exactly the ones the service sampled, and a rank the
service's LoRA kernels support.
"""

from __future__ import annotations

import math
from collections.abc import Mapping
from dataclasses import dataclass

SUPPORTED_LORA_RANKS = (8, 16, 32, 64, 128)
_KEYS = ("rank", "alpha", "layers")


def _distinct_indices(values) -> bool:
    return (isinstance(values, tuple) and len(values) > 0 and len(set(values)) == len(values)
            and all(type(v) is int and v >= 0 for v in values))


def parse_lora_layers(value: str) -> tuple[int, ...] | None:
    """``"all"`` (every layer, returned as None) or comma-separated distinct layer indices."""
    if not isinstance(value, str):
        raise ValueError("LoRA layers must be 'all' or comma-separated layer indices")
    text = value.strip()
    if text == "all":
        return None
    items = [item.strip() for item in text.split(",")]
    if not all(item.isascii() and item.isdigit() for item in items):
        raise ValueError("LoRA layers must be 'all' or comma-separated nonnegative indices")
    layers = tuple(int(item) for item in items)
    if len(set(layers)) < len(layers):
        raise ValueError("LoRA layer indices must be distinct")
    return tuple(sorted(layers))


@dataclass(frozen=True)
class DistributedLoRAConfig:
    rank: int = 8
    alpha: float = 8.0
    layers: tuple[int, ...] | None = None

    def __post_init__(self):
        if not (type(self.rank) is int and self.rank in SUPPORTED_LORA_RANKS):
            raise ValueError(f"LoRA rank must be one of {SUPPORTED_LORA_RANKS}")
        alpha = self.alpha
        if not (type(alpha) in (int, float) and math.isfinite(alpha) and alpha > 0):
            raise ValueError("LoRA alpha must be finite and positive")
        object.__setattr__(self, "alpha", float(alpha))
        if self.layers is not None:
            if not _distinct_indices(self.layers):
                raise ValueError("LoRA layers must be distinct nonnegative indices or None")
            object.__setattr__(self, "layers", tuple(sorted(self.layers)))

    def selected_layers(self, num_layers: int) -> tuple[int, ...]:
        if not (type(num_layers) is int and num_layers >= 1):
            raise ValueError("backbone layer count must be a positive integer")
        chosen = self.layers if self.layers is not None else tuple(range(num_layers))
        if max(chosen) >= num_layers:
            raise ValueError(f"LoRA layer index is outside the {num_layers}-layer backbone")
        return chosen

    def parameter_count(self, hidden: int, q_rank: int, num_layers: int) -> int:
        """A [rank, hidden] and B [q_rank, rank] per selected layer."""
        if not all(type(n) is int and n >= 1 for n in (hidden, q_rank)):
            raise ValueError("query projection dimensions must be positive integers")
        return len(self.selected_layers(num_layers)) * self.rank * (hidden + q_rank)

    def to_dict(self) -> dict:
        return {"rank": self.rank, "alpha": self.alpha, "layers": None if self.layers is None else list(self.layers)}

    @classmethod
    def from_dict(cls, value: Mapping) -> "DistributedLoRAConfig":
        if not isinstance(value, Mapping) or set(value) != set(_KEYS):
            raise ValueError("LoRA configuration requires exactly rank, alpha and layers")
        layers = value["layers"]
        if not (layers is None or isinstance(layers, list)):
            raise ValueError("serialized LoRA layers must be a list or null")
        return cls(rank=value["rank"], alpha=value["alpha"], layers=None if layers is None else tuple(layers))

    def lora_config(self):
        """The learner-side ``LoRAConfig``: the query down-projection only, no dropout."""
        from ..lora import LoRAConfig

        return LoRAConfig(self.rank, self.alpha, 0.0, ("attention.q_a",))


__all__ = ["DistributedLoRAConfig", "SUPPORTED_LORA_RANKS", "parse_lora_layers"]
