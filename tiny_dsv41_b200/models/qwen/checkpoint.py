"""Hugging Face ``Qwen3-MoE`` safetensors <-> the native model.

HF stores every expert projection as its own tensor
(``model.layers.N.mlp.experts.E.{gate,up,down}_proj.weight``); the native model keeps one
stacked ``gate_up_proj [E_local, 2I, H]`` (gate rows first, then up rows) and
``down_proj [E_local, H, I]`` per layer, holding only this EP rank's experts
(``dsv41_train/models/qwen/checkpoint.py:17-187`` defines the same mapping).

Loading streams tensor by tensor from the memory-mapped shards straight into the target
parameters (``load_qwen3_moe``), so peak host memory is one model copy, and an EP rank reads
only its own experts' bytes.
"""

from __future__ import annotations

import json
import re
from pathlib import Path

import torch

from ...utils.safetensors_io import ShardedSafeTensorReader, save_sharded
from .config import Qwen3MoeConfig
from .model import Qwen3MoeExperts, Qwen3MoeForCausalLM

_EXPERT = re.compile(r"^(model\.layers\.\d+\.mlp\.experts)\.(\d+)\.(gate_proj|up_proj|down_proj)\.weight$")


def hf_tensor_names(config: Qwen3MoeConfig) -> list[str]:
    names = ["model.embed_tokens.weight", "model.norm.weight", "lm_head.weight"]
    for i in range(config.num_hidden_layers):
        p = f"model.layers.{i}."
        names += [p + n for n in ("self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
                                  "self_attn.o_proj.weight", "self_attn.q_norm.weight", "self_attn.k_norm.weight",
                                  "input_layernorm.weight", "post_attention_layernorm.weight", "mlp.gate.weight")]
        names += [f"{p}mlp.experts.{e}.{proj}.weight" for e in range(config.num_experts)
                  for proj in ("gate_proj", "up_proj", "down_proj")]
    return names


@torch.no_grad()
def load_qwen3_moe(folder, *, device="cpu", dtype=torch.bfloat16, context_parallel=None,
                   token_dispatcher=None) -> Qwen3MoeForCausalLM:
    """Build the native model from an HF Qwen3-MoE folder (config.json + safetensors shards)."""
    folder = Path(folder)
    config = Qwen3MoeConfig.from_json(folder / "config.json")
    with torch.device("meta"):
        model = Qwen3MoeForCausalLM(config, context_parallel, token_dispatcher)
    model.to_empty(device=device)
    if dtype is not None:
        model.to(dtype)
    params = dict(model.named_parameters())
    experts = {name: m for name, m in model.named_modules() if isinstance(m, Qwen3MoeExperts)}
    seen: set[str] = set()
    filled: dict[str, int] = {}
    with ShardedSafeTensorReader(folder) as reader:
        for name in sorted(reader.weight_map):
            match = _EXPERT.fullmatch(name)
            if match is None:
                if name not in params:
                    raise ValueError(f"unexpected checkpoint tensor: {name}")
                value = reader.tensor(name)
                if tuple(value.shape) != tuple(params[name].shape):
                    raise ValueError(f"shape mismatch for {name}: {tuple(value.shape)}")
                params[name].copy_(value)
                seen.add(name)
                continue
            prefix, expert, proj = match.groups()
            module = experts.get(prefix)
            if module is None:
                raise ValueError(f"checkpoint has experts for a layer without them: {prefix}")
            local = int(expert) - module.expert_start
            if not 0 <= int(expert) < config.num_experts:
                raise ValueError(f"expert id out of range: {name}")
            if not 0 <= local < module.num_experts:
                continue  # another EP rank's expert
            value = reader.tensor(name)
            inter = module.intermediate_size
            if proj == "gate_proj":
                module.gate_up_proj[local, :inter].copy_(value)
            elif proj == "up_proj":
                module.gate_up_proj[local, inter:].copy_(value)
            else:
                module.down_proj[local].copy_(value)
            filled[prefix] = filled.get(prefix, 0) + 1
    missing = [n for n in params if n not in seen and not any(n.startswith(p + ".") for p in experts)]
    if missing:
        raise ValueError(f"checkpoint is missing tensors: {missing[:5]}")
    for prefix, module in experts.items():
        if filled.get(prefix, 0) != 3 * module.num_experts:
            raise ValueError(f"checkpoint has incomplete experts for {prefix}")
    return model


@torch.no_grad()
def save_qwen3_moe(model: Qwen3MoeForCausalLM, folder, shard_size: int = 2 ** 30) -> None:
    """Write a single-rank native model in the HF layout (config.json + sharded safetensors)."""
    folder = Path(folder)
    folder.mkdir(parents=True, exist_ok=True)
    out: dict[str, torch.Tensor] = {}
    experts = {name: m for name, m in model.named_modules() if isinstance(m, Qwen3MoeExperts)}
    for name, value in model.state_dict().items():
        owner = next((p for p in experts if name.startswith(p + ".")), None)
        if owner is None:
            out[name] = value.detach().cpu().contiguous()
            continue
        module = experts[owner]
        if module.num_experts != model.config.num_experts:
            raise ValueError("save_qwen3_moe needs all experts on this rank")
        inter = module.intermediate_size
        for e in range(module.num_experts):
            if name.endswith("gate_up_proj"):
                out[f"{owner}.{e}.gate_proj.weight"] = value[e, :inter].detach().cpu().contiguous()
                out[f"{owner}.{e}.up_proj.weight"] = value[e, inter:].detach().cpu().contiguous()
            else:
                out[f"{owner}.{e}.down_proj.weight"] = value[e].detach().cpu().contiguous()
    save_sharded(out, folder, shard_size)
    (folder / "config.json").write_text(json.dumps(model.config.to_dict(), indent=2), encoding="utf-8")


__all__ = ["hf_tensor_names", "load_qwen3_moe", "save_qwen3_moe"]
