"""Low-rank adapters (LoRA) on linear projections, and the adapter file.

Interface and on-disk format shared with ``dsv41_train/lora.py`` (adapters trained by either side
load in the other, and the RL packet exporter reads them):

* ``LoRAConfig(rank, alpha, dropout, targets)``; targets are exact module paths or dotted suffixes.
* ``adapter.pt`` = ``{"format_version": 1 | 2, "layer_ids": [...], "base_identity": {...} (v2 only),
  "modules": {path: asdict(LoRAConfig)}, "weights": {path.lora_a / path.lora_b: tensor}}``.
  Version 2 binds the adapter to its base model (weights and tokenizer identity); version 1 files
  load with a warning and architecture-only checks.

``LoRALinear`` keeps the frozen base weight W, A [rank, in] (Kaiming-uniform) and B [out, rank]
(zeros): y = x W^T + scale * (x A^T) B^T with scale = alpha / rank. All three products run on this
library's tcgen05 GEMM. Merging folds scale * B A into W for inference (in fp32 for 16-bit
weights); the state dict always holds the unmerged W. Adapters are injected after the base weights
are loaded and before FSDP wraps the model.
"""

from __future__ import annotations

import json
import math
import warnings
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Iterator

import torch
import torch.distributed as dist
from torch import nn

from . import ops
from .models.common import Linear

FORMAT_LEGACY, FORMAT_BOUND = 1, 2
_ADAPTER_LEAVES = ("lora_a", "lora_b")


def _require(condition: bool, message: str) -> None:
    if not condition:
        raise ValueError(message)


@dataclass(frozen=True)
class LoRAConfig:
    rank: int = 8
    alpha: float = 16.0
    dropout: float = 0.0
    targets: tuple[str, ...] = ("attention.q_a", "attention.q_b", "attention.kv_proj", "attention.o_b")

    def __post_init__(self):
        _require(type(self.rank) is int and self.rank >= 1, "LoRA rank must be a positive integer")
        _require(math.isfinite(self.alpha) and self.alpha > 0, "LoRA alpha must be positive and finite")
        _require(0 <= self.dropout < 1, "LoRA dropout must be in [0, 1)")
        names = self.targets
        _require(isinstance(names, (tuple, list)) and len(names) > 0 and all(isinstance(n, str) and n for n in names),
                 "LoRA targets must contain module names")
        object.__setattr__(self, "targets", tuple(names))

    @property
    def scaling(self) -> float:
        return self.alpha / self.rank


def _plain_linear(module: nn.Module) -> nn.Linear:
    _require(isinstance(module, nn.Linear), "LoRA only supports nn.Linear targets")
    _require(not module.weight.is_meta and not hasattr(module.weight, "to_local"),
             "inject LoRA after loading and before FSDP wrapping")
    return module


def _unsharded(weight: torch.Tensor) -> bool:
    return not weight.is_meta and not hasattr(weight, "to_local")


class LoRALinear(Linear):
    def __init__(self, base: nn.Linear, config: LoRAConfig):
        base = _plain_linear(base)
        nn.Module.__init__(self)
        self.in_features, self.out_features = base.in_features, base.out_features
        self.weight, self.bias = base.weight.requires_grad_(False), base.bias
        if self.bias is not None:
            self.bias.requires_grad_(False)
        self.config = config
        self.scaling = config.scaling
        self.adapters_enabled = True
        self.lora_a = nn.Parameter(base.weight.new_empty(config.rank, self.in_features))
        nn.init.kaiming_uniform_(self.lora_a, a=math.sqrt(5))
        self.lora_b = nn.Parameter(base.weight.new_zeros(self.out_features, config.rank))
        self.dropout = nn.Dropout(config.dropout)
        # while merged, the original W (what the state dict and unmerge return to)
        self.register_buffer("_unmerged_weight", None, persistent=False)
        self.train(base.training)

    @property
    def merged(self) -> bool:
        return self._unmerged_weight is not None

    def _adapter_delta(self, x: torch.Tensor) -> torch.Tensor:
        down = ops.linear(self.dropout(x), self.lora_a.to(x.dtype))
        return ops.linear(down, self.lora_b.to(x.dtype)) * self.scaling

    def forward(self, x):
        use_adapter = self.adapters_enabled and not self.merged
        weight = self._unmerged_weight if (self.merged and not self.adapters_enabled) else self.weight
        y = ops.linear(x, weight)
        if self.bias is not None:
            y = y + self.bias.to(y.dtype)
        return y + self._adapter_delta(x) if use_adapter else y

    def train(self, mode=True):
        if mode:
            self.unmerge()  # training always sees W and the adapter separately
        return super().train(mode)

    def _save_to_state_dict(self, destination, prefix, keep_vars):
        super()._save_to_state_dict(destination, prefix, keep_vars)
        if self.merged:
            destination[prefix + "weight"] = self._unmerged_weight if keep_vars else self._unmerged_weight.detach()

    def _load_from_state_dict(self, *args, **kwargs):
        self.unmerge()
        super()._load_from_state_dict(*args, **kwargs)

    @torch.no_grad()
    def merge(self):
        _require(_unsharded(self.weight) and not self.training,
                 "merge requires a materialized, unsharded model in eval mode")
        if self.merged:
            return
        self._unmerged_weight = self.weight.detach().clone()
        wide = torch.float32 if self.weight.dtype in (torch.float16, torch.bfloat16) else self.weight.dtype
        delta = (self.lora_b.to(wide) @ self.lora_a.to(wide)) * self.scaling
        self.weight.copy_((self.weight.to(wide) + delta).to(self.weight.dtype))

    @torch.no_grad()
    def unmerge(self):
        if self.merged:
            self.weight.copy_(self._unmerged_weight)
            self._unmerged_weight = None


# -- injection ------------------------------------------------------------------------------------
def _matching(modules: dict[str, nn.Module], target: str) -> dict[str, nn.Module]:
    suffix = "." + target
    return {name: m for name, m in modules.items() if name == target or name.endswith(suffix)}


def inject_lora(model: nn.Module, config: LoRAConfig) -> list[str]:
    """Replace every target projection by a ``LoRALinear`` and freeze everything else. Returns the
    wrapped module paths."""
    _require(not any(isinstance(m, LoRALinear) for m in model.modules()), "LoRA is already installed")
    modules = dict(model.named_modules())
    chosen: dict[str, nn.Module] = {}
    for target in config.targets:
        found = _matching(modules, target)
        _require(bool(found), f"LoRA target did not match a module: {target}")
        chosen.update((name, _plain_linear(m)) for name, m in found.items())
    model.requires_grad_(False)
    for path, base in chosen.items():
        parent, _, leaf = path.rpartition(".")
        setattr(model.get_submodule(parent), leaf, LoRALinear(base, config))
    return list(chosen)


def adapter_parameters(model: nn.Module) -> Iterator[nn.Parameter]:
    for module in model.modules():
        if isinstance(module, LoRALinear):
            yield from (module.lora_a, module.lora_b)


def _adapters(model: nn.Module) -> dict[str, LoRALinear]:
    found = {name: m for name, m in model.named_modules() if isinstance(m, LoRALinear)}
    _require(bool(found), "model has no LoRA adapters")
    return found


def _join(*parts: str) -> str:
    return ".".join(p for p in parts if p)


def _layer_ids(model: nn.Module):
    """The decoder layers the model holds (a window of a larger checkpoint keeps its own ids)."""
    decoder = getattr(model, "model", None)
    if hasattr(decoder, "layer_ids"):
        return decoder.layer_ids
    layers = getattr(decoder, "layers", None)
    if layers is None:
        return None
    return [getattr(layer, "layer_id", index) for index, layer in enumerate(layers)]


# -- the adapter file -----------------------------------------------------------------------------
def _canonical_identity(identity) -> dict:
    _require(isinstance(identity, dict) and len(identity) > 0, "adapter base identity must be a nonempty object")
    try:
        return json.loads(json.dumps(identity, sort_keys=True, allow_nan=False))
    except (TypeError, ValueError) as error:
        raise ValueError("adapter base identity must contain JSON metadata") from error


def _check_binding(payload: dict, expected) -> None:
    version = payload["format_version"]
    if version == FORMAT_LEGACY:
        warnings.warn("Legacy adapter v1 has no base identity: base weights and tokenizer cannot be verified; "
                      "loading with architecture-only validation.", RuntimeWarning, stacklevel=3)
        return
    _require(version == FORMAT_BOUND, "unsupported adapter format")
    _require(expected is not None and _canonical_identity(payload["base_identity"]) == _canonical_identity(expected),
             "adapter base identity differs or was not provided")


def _payload_keys(version: int) -> set[str]:
    keys = {"format_version", "layer_ids", "modules", "weights"}
    return keys | {"base_identity"} if version == FORMAT_BOUND else keys


@torch.no_grad()
def save_adapter(model: nn.Module, path, *, base_identity=None):
    """Every rank takes part (sharded adapters are gathered); rank zero writes the file."""
    adapters = _adapters(model)
    is_writer = not dist.is_initialized() or dist.get_rank() == 0
    weights = {}
    for name, module in adapters.items():
        for leaf in _ADAPTER_LEAVES:
            tensor = getattr(module, leaf).detach()
            tensor = tensor.full_tensor() if hasattr(tensor, "full_tensor") else tensor  # collective
            if is_writer:
                weights[_join(name, leaf)] = tensor.cpu()
    if not is_writer:
        return
    payload = {"format_version": FORMAT_LEGACY if base_identity is None else FORMAT_BOUND,
               "layer_ids": _layer_ids(model)}
    if base_identity is not None:
        payload["base_identity"] = _canonical_identity(base_identity)
    payload["modules"] = {name: asdict(module.config) for name, module in adapters.items()}
    payload["weights"] = weights
    target = Path(path)
    target.parent.mkdir(parents=True, exist_ok=True)
    torch.save(payload, target)


def read_adapter(path, *, base_identity=None) -> dict:
    payload = torch.load(path, map_location="cpu", weights_only=True)
    version = payload.get("format_version") if isinstance(payload, dict) else None
    _require(version in (FORMAT_LEGACY, FORMAT_BOUND), "unsupported adapter format")
    well_formed = (set(payload) == _payload_keys(version) and isinstance(payload["modules"], dict)
                   and isinstance(payload["weights"], dict)
                   and all(isinstance(n, str) for n in (*payload["modules"], *payload["weights"])))
    _require(well_formed, "invalid adapter payload")
    if version == FORMAT_BOUND:
        _canonical_identity(payload["base_identity"])
        if base_identity is not None:
            _check_binding(payload, base_identity)
    return payload


def validate_adapter_layout(model: nn.Module, payload: dict):
    _require(payload.get("layer_ids") == _layer_ids(model), "adapter layer window does not match the current model")


def _comparable(config: dict) -> dict:
    # configs come back from torch.load with lists where the dataclass holds tuples
    return {key: tuple(value) if isinstance(value, list) else value for key, value in config.items()}


@torch.no_grad()
def load_adapter_state(model: nn.Module, payload: dict, *, prefix: str = "", base_identity=None):
    """Copy the adapter tensors of ``payload`` (below ``prefix``) into the model's adapters after
    checking binding, configuration, names, shapes and finiteness - nothing is written unless
    every check passes."""
    _check_binding(payload, base_identity)
    adapters = {_join(prefix, name): m for name, m in _adapters(model).items()}
    scope = prefix + "." if prefix else ""
    in_scope = lambda name: name == prefix or name.startswith(scope)  # noqa: E731
    stored = {n: _comparable(c) for n, c in payload["modules"].items() if in_scope(n)}
    _require(stored == {n: _comparable(asdict(m.config)) for n, m in adapters.items()},
             "adapter configuration does not match the current model")
    targets = {_join(name, leaf): getattr(m, leaf) for name, m in adapters.items() for leaf in _ADAPTER_LEAVES}
    incoming = {n: t for n, t in payload["weights"].items() if n.startswith(scope)}
    _require(incoming.keys() == targets.keys(), "adapter tensor names do not match")
    _require(not any(m.merged for m in adapters.values()), "unmerge adapters before loading")
    for name, target in targets.items():
        value = incoming[name]
        _require(_unsharded(target), "load adapters after materialization and before FSDP wrapping")
        _require(isinstance(value, torch.Tensor) and value.shape == target.shape,
                 f"adapter tensor shape does not match: {name}")
        _require(value.layout == torch.strided and value.is_floating_point() and bool(torch.isfinite(value).all()),
                 f"adapter tensor must contain finite floating values: {name}")
    for name, target in targets.items():
        target.copy_(incoming[name])


def load_adapter(model: nn.Module, path, *, base_identity=None):
    payload = read_adapter(path, base_identity=base_identity)
    validate_adapter_layout(model, payload)
    load_adapter_state(model, payload, base_identity=base_identity)


def merge_adapters(model: nn.Module):
    adapters = _adapters(model).values()
    _require(all(not m.training and _unsharded(m.weight) for m in adapters),
             "merge requires a materialized, unsharded model in eval mode")
    for module in adapters:
        module.merge()


def unmerge_adapters(model: nn.Module):
    for module in _adapters(model).values():
        module.unmerge()


__all__ = ["LoRAConfig", "LoRALinear", "adapter_parameters", "inject_lora", "load_adapter", "load_adapter_state",
           "merge_adapters", "read_adapter", "save_adapter", "unmerge_adapters", "validate_adapter_layout"]
