"""Single-process layer placement for one RL policy (``dsv41_train/rl/parallel.py:7-42``).

``layer_device_map`` assigns contiguous decoder layers to the listed devices; a policy then runs
its layers in order, moving the hidden state between devices (sequential, no micro-batching).
"""

from __future__ import annotations

import torch
from torch import nn


def layer_device_map(num_layers: int, devices) -> tuple[torch.device, ...]:
    devices = tuple(torch.device(d) for d in devices)
    if not devices or len(devices) > num_layers:
        raise ValueError("use between one device and num_hidden_layers devices per policy")
    if any(d.type == "cpu" for d in devices):
        if devices != (torch.device("cpu"),):
            raise ValueError("CPU execution requires exactly one device")
    elif any(d.type != "cuda" or d.index is None for d in devices):
        raise ValueError("use cpu or explicit CUDA device indices")
    if len(set(devices)) != len(devices):
        raise ValueError("policy devices must not contain duplicates")
    return tuple(devices[i * len(devices) // num_layers] for i in range(num_layers))


def validate_available_devices(devices) -> None:
    for value in devices:
        device = torch.device(value)
        if device.type == "cuda" and (not torch.cuda.is_available() or device.index >= torch.cuda.device_count()):
            count = torch.cuda.device_count() if torch.cuda.is_available() else 0
            raise ValueError(f"{device} is unavailable; CUDA exposes {count} devices")


def _move(value, device):
    if isinstance(value, torch.Tensor):
        return value.to(device)
    if isinstance(value, tuple):
        return tuple(_move(v, device) for v in value)
    if isinstance(value, list):
        return [_move(v, device) for v in value]
    if isinstance(value, dict):
        return {k: _move(v, device) for k, v in value.items()}
    return value


def pin_inputs_to(module: nn.Module, device: torch.device):
    """Forward pre-hook that moves every tensor argument of ``module`` to ``device``."""
    def hook(_module, args, kwargs):
        return _move(args, device), _move(kwargs, device)

    return module.register_forward_pre_hook(hook, with_kwargs=True)


__all__ = ["layer_device_map", "pin_inputs_to", "validate_available_devices"]
