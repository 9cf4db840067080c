"""LoRA adapters on linear projections, with the reference's adapter file format.

API and on-disk format of ``dsv41_train/lora.py``: ``LoRAConfig(rank, alpha, dropout, targets)``,
``inject_lora`` (exact module paths or dotted suffixes, before FSDP), ``LoRALinear`` (A kaiming,
B zeros, scale alpha/rank, merge/unmerge keeping W/A/B in the state dict), ``save_adapter`` /
``read_adapter`` / ``load_adapter`` / ``validate_adapter_layout`` with ``adapter.pt`` =
``{format_version 1|2, layer_ids, [base_identity], modules{name: config}, weights{name.lora_a/b}}``.

The base projection runs on the tcgen05 GEMM; the adapter path is two thin GEMMs on the same kernel.
"""

from __future__ import annotations

import json
import math
import warnings
from dataclasses import asdict, dataclass
from pathlib import Path

import torch
import torch.distributed as dist
from torch import nn

from . import ops
from .models.common import Linear


@dataclass(frozen=True)
class LoRAConfig:
    rank: int = 8
    alpha: float = 16.0
    dropout: float = 0.0
    targets: tuple[str, ...] = ("attention.q_a", "attention.q_b", "attention.kv_proj", "attention.o_b")

    def __post_init__(self):
        if type(self.rank) is not int or self.rank < 1:
            raise ValueError("LoRA rank must be a positive integer")
        if not math.isfinite(self.alpha) or self.alpha <= 0:
            raise ValueError("LoRA alpha must be positive and finite")
        if not 0 <= self.dropout < 1:
            raise ValueError("LoRA dropout must be in [0, 1)")
        if (not isinstance(self.targets, (tuple, list)) or not self.targets
                or any(not isinstance(n, str) or not n for n in self.targets)):
            raise ValueError("LoRA targets must contain module names")
        object.__setattr__(self, "targets", tuple(self.targets))


def _check_linear(module):
    if not isinstance(module, nn.Linear):
        raise ValueError("LoRA only supports nn.Linear targets")
    if module.weight.is_meta or hasattr(module.weight, "to_local"):
        raise ValueError("inject LoRA after loading and before FSDP wrapping")


class LoRALinear(Linear):
    def __init__(self, base: nn.Linear, config: LoRAConfig):
        _check_linear(base)
        nn.Module.__init__(self)
        self.in_features, self.out_features = base.in_features, base.out_features
        self.weight, self.bias = base.weight, base.bias
        self.weight.requires_grad_(False)
        if self.bias is not None:
            self.bias.requires_grad_(False)
        self.config = config
        self.scaling = config.alpha / config.rank
        self.adapters_enabled = True
        self.lora_a = nn.Parameter(base.weight.new_empty(config.rank, self.in_features))
        self.lora_b = nn.Parameter(base.weight.new_zeros(self.out_features, config.rank))
        nn.init.kaiming_uniform_(self.lora_a, a=math.sqrt(5))
        self.dropout = nn.Dropout(config.dropout)
        self.register_buffer("_unmerged_weight", None, persistent=False)
        self.train(base.training)

    @property
    def merged(self) -> bool:
        return self._unmerged_weight is not None

    def forward(self, x):
        weight = self._unmerged_weight if self.merged and not self.adapters_enabled else self.weight
        out = ops.linear(x, weight)
        if self.bias is not None:
            out = out + self.bias.to(out.dtype)
        if self.adapters_enabled and not self.merged:
            low = ops.linear(self.dropout(x), self.lora_a.to(x.dtype))
            out = out + ops.linear(low, self.lora_b.to(x.dtype)) * self.scaling
        return out

    def train(self, mode=True):
        if mode and self.merged:
            self.unmerge()
        return super().train(mode)

    def _save_to_state_dict(self, destination, prefix, keep_vars):
        super()._save_to_state_dict(destination, prefix, keep_vars)
        if self.merged:
            weight = self._unmerged_weight
            destination[prefix + "weight"] = weight if keep_vars else weight.detach()

    def _load_from_state_dict(self, *args, **kwargs):
        self.unmerge()
        super()._load_from_state_dict(*args, **kwargs)

    @torch.no_grad()
    def merge(self):
        if hasattr(self.weight, "to_local") or self.weight.is_meta or self.training:
            raise ValueError("merge requires a materialized, unsharded model in eval mode")
        if not self.merged:
            self._unmerged_weight = self.weight.detach().clone()
            dtype = torch.float32 if self.weight.dtype in (torch.float16, torch.bfloat16) else self.weight.dtype
            delta = self.lora_b.to(dtype) @ self.lora_a.to(dtype)
            self.weight.copy_((self.weight.to(dtype) + delta * self.scaling).to(self.weight.dtype))

    @torch.no_grad()
    def unmerge(self):
        if self.merged:
            self.weight.copy_(self._unmerged_weight)
            self._unmerged_weight = None


def inject_lora(model: nn.Module, config: LoRAConfig) -> list[str]:
    if any(isinstance(m, LoRALinear) for m in model.modules()):
        raise ValueError("LoRA is already installed")
    selected = {}
    modules = dict(model.named_modules())
    for target in config.targets:
        matches = {n: m for n, m in modules.items() if n == target or n.endswith("." + target)}
        if not matches:
            raise ValueError(f"LoRA target did not match a module: {target}")
        for m in matches.values():
            _check_linear(m)
        selected.update(matches)
    model.requires_grad_(False)
    for name, module in selected.items():
        parent, _, leaf = name.rpartition(".")
        setattr(model.get_submodule(parent), leaf, LoRALinear(module, config))
    return list(selected)


def adapter_parameters(model: nn.Module):
    for m in model.modules():
        if isinstance(m, LoRALinear):
            yield m.lora_a
            yield m.lora_b


def _adapter_modules(model):
    modules = {n: m for n, m in model.named_modules() if isinstance(m, LoRALinear)}
    if not modules:
        raise ValueError("model has no LoRA adapters")
    return modules


def _key(name, leaf):
    return ".".join(p for p in (name, leaf) if p)


def _layer_ids(model):
    decoder = getattr(model, "model", None)
    if hasattr(decoder, "layer_ids"):
        return decoder.layer_ids
    if hasattr(decoder, "layers"):
        return [getattr(layer, "layer_id", i) for i, layer in enumerate(decoder.layers)]
    return None


def _base_identity(identity):
    if not isinstance(identity, dict) or not identity:
        raise ValueError("adapter base identity must be a nonempty object")
    try:
        return json.loads(json.dumps(identity, sort_keys=True, allow_nan=False))
    except (TypeError, ValueError) as error:
        raise ValueError("adapter base identity must contain JSON metadata") from error


def _validate_adapter_base(payload, expected):
    if payload["format_version"] == 1:
        warnings.warn("Legacy adapter v1 has no base identity: base weights and tokenizer cannot be verified; "
                      "loading with architecture-only validation.", RuntimeWarning, stacklevel=3)
    elif payload["format_version"] != 2:
        raise ValueError("unsupported adapter format")
    elif expected is None or _base_identity(payload["base_identity"]) != _base_identity(expected):
        raise ValueError("adapter base identity differs or was not provided")


@torch.no_grad()
def save_adapter(model: nn.Module, path, *, base_identity=None):
    """All ranks participate (DTensor adapters are gathered); rank zero writes."""
    binding = {} if base_identity is None else {"base_identity": _base_identity(base_identity)}
    modules = _adapter_modules(model)
    writer = not dist.is_initialized() or dist.get_rank() == 0
    weights = {}
    for name, module in modules.items():
        for key in ("lora_a", "lora_b"):
            value = getattr(module, key).detach()
            if hasattr(value, "full_tensor"):
                value = value.full_tensor()
            if writer:
                weights[_key(name, key)] = value.cpu()
    if writer:
        path = Path(path)
        path.parent.mkdir(parents=True, exist_ok=True)
        torch.save({"format_version": 2 if binding else 1, "layer_ids": _layer_ids(model), **binding,
                    "modules": {n: asdict(m.config) for n, m in modules.items()}, "weights": weights}, path)


def read_adapter(path, *, base_identity=None) -> dict:
    payload = torch.load(path, map_location="cpu", weights_only=True)
    if not isinstance(payload, dict) or payload.get("format_version") not in (1, 2):
        raise ValueError("unsupported adapter format")
    expected = {"format_version", "layer_ids", "modules", "weights"}
    if payload["format_version"] == 2:
        expected.add("base_identity")
    if (set(payload) != expected or not isinstance(payload["modules"], dict) or not isinstance(payload["weights"], dict)
            or any(not isinstance(n, str) for n in (*payload["modules"], *payload["weights"]))):
        raise ValueError("invalid adapter payload")
    if payload["format_version"] == 2:
        _base_identity(payload["base_identity"])
        if base_identity is not None:
            _validate_adapter_base(payload, base_identity)
    return payload


def validate_adapter_layout(model: nn.Module, payload: dict):
    if payload.get("layer_ids") != _layer_ids(model):
        raise ValueError("adapter layer window does not match the current model")


@torch.no_grad()
def load_adapter_state(model: nn.Module, payload: dict, *, prefix: str = "", base_identity=None):
    _validate_adapter_base(payload, base_identity)
    modules = {_key(prefix, n): m for n, m in _adapter_modules(model).items()}
    namespace = prefix + "." if prefix else ""
    expected = {n: asdict(m.config) for n, m in modules.items()}
    metadata = {n: v for n, v in payload["modules"].items() if n == prefix or n.startswith(namespace)}
    # configs round-trip through torch.save as dicts; targets may come back as lists
    norm = lambda d: {k: (tuple(v) if isinstance(v, list) else v) for k, v in d.items()}  # noqa: E731
    if {n: norm(v) for n, v in metadata.items()} != {n: norm(v) for n, v in expected.items()}:
        raise ValueError("adapter configuration does not match the current model")
    targets = {_key(n, k): getattr(m, k) for n, m in modules.items() for k in ("lora_a", "lora_b")}
    weights = {n: v for n, v in payload["weights"].items() if n.startswith(namespace)}
    if weights.keys() != targets.keys():
        raise ValueError("adapter tensor names do not match")
    if any(m.merged for m in modules.values()):
        raise ValueError("unmerge adapters before loading")
    for name, target in targets.items():
        value = weights[name]
        if target.is_meta or hasattr(target, "to_local"):
            raise ValueError("load adapters after materialization and before FSDP wrapping")
        if not isinstance(value, torch.Tensor) or value.shape != target.shape:
            raise ValueError(f"adapter tensor shape does not match: {name}")
        if value.layout != torch.strided or not value.is_floating_point() or not torch.isfinite(value).all():
            raise ValueError(f"adapter tensor must contain finite floating values: {name}")
    for name, target in targets.items():
        target.copy_(weights[name])


def load_adapter(model: nn.Module, path, *, base_identity=None):
    payload = read_adapter(path, base_identity=base_identity)
    validate_adapter_layout(model, payload)
    load_adapter_state(model, payload, base_identity=base_identity)


def merge_adapters(model: nn.Module):
    modules = _adapter_modules(model)
    if any(m.training or m.weight.is_meta or hasattr(m.weight, "to_local") for m in modules.values()):
        raise ValueError("merge requires a materialized, unsharded model in eval mode")
    for m in modules.values():
        m.merge()


def unmerge_adapters(model: nn.Module):
    for m in _adapter_modules(model).values():
        m.unmerge()


__all__ = ["LoRAConfig", "LoRALinear", "adapter_parameters", "inject_lora", "load_adapter", "load_adapter_state",
           "merge_adapters", "read_adapter", "save_adapter", "unmerge_adapters", "validate_adapter_layout"]
