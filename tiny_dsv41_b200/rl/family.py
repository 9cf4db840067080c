"""Which model family an RL run trains, and how its policy is built.

The selection rules follow ``dsv41_train/rl/family.py:11-99``: a flat, unquantized
``config.json`` with ``model_type == "qwen3_moe"`` is a Qwen3-MoE policy; ``deepseek_v41``,
``deepseek_v41_text`` or no type (at the root or in ``text_config``) is DeepSeek-V4.1. Anything
else is refused before a model is built.
"""

from __future__ import annotations

import json
from dataclasses import asdict
from pathlib import Path

from ..lora import LoRAConfig
from .policy import build_dsv41_policy, build_qwen_policy, validate_qwen_config

QWEN = "qwen3_moe"
DSV4_TYPES = (None, "deepseek_v41", "deepseek_v41_text")
QWEN_LORA_TARGETS = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj")


def is_qwen(model_config) -> bool:
    return getattr(model_config, "model_type", None) == QWEN


def policy_lora_config(config, model_config):
    """The adapter configuration of a ``trainable_scope="lora"`` run (None otherwise); the default
    targets depend on the family."""
    if config.trainable_scope != "lora":
        return None
    default = QWEN_LORA_TARGETS if is_qwen(model_config) else LoRAConfig().targets
    return LoRAConfig(config.lora_rank, config.lora_alpha, config.lora_dropout, config.lora_targets or default)


def lora_metadata(lora_config, initial_adapter) -> dict:
    from .checkpoint import file_sha256

    adapter_hash = file_sha256(initial_adapter) if initial_adapter else None
    return json.loads(json.dumps({"config": asdict(lora_config), "initial_adapter_sha256": adapter_hash}))


def initial_sft_source(model_dir, model_config, config, random_init):
    """The full-SFT snapshot named by ``initial_sft_checkpoint`` (DeepSeek with a pretrained base)."""
    if config.initial_sft_checkpoint is None:
        return None
    if random_init or is_qwen(model_config):
        raise ValueError("initial_sft_checkpoint requires a pretrained DSV4 base")
    from ..train.sft_source import SFTCheckpointSource

    return SFTCheckpointSource(config.initial_sft_checkpoint, model_dir)


def _load_qwen(path: Path, values: dict):
    if values.get("text_config") is not None:
        raise ValueError("native Qwen RL requires a flat qwen3_moe config")
    if values.get("quantization_config"):
        raise ValueError("native Qwen RL requires unquantized mounted safetensors")
    from ..models.qwen import Qwen3MoeConfig

    config = Qwen3MoeConfig.from_json(path)
    validate_qwen_config(config)
    return config


def _load_deepseek(path: Path, values: dict, text: dict):
    from ..models.dsv4.config import DeepSeekV41Config

    config = DeepSeekV41Config.from_json(path)
    quantized = bool(values.get("quantization_config") or text.get("quantization_config"))
    layout = values.get("checkpoint_format", "released" if quantized else "native")
    layout = "native" if layout == "tiny_dsv41" else layout
    if layout not in ("native", "released"):
        raise ValueError("DeepSeek checkpoint_format must be native or released")
    config.checkpoint_format = layout
    if config.attention_dropout:
        raise ValueError("RL policies require attention_dropout=0 for behavior probability consistency")
    return config


def load_model_config(model_dir):
    path = Path(model_dir) / "config.json"
    values = json.loads(path.read_text(encoding="utf-8"))
    if not isinstance(values, dict):
        raise ValueError("model config must be an object")
    text = values.get("text_config")
    if not (text is None or isinstance(text, dict)):
        raise ValueError("text_config must be an object")
    text = text or {}
    root_type, text_type = values.get("model_type"), text.get("model_type")
    if root_type == QWEN:
        return _load_qwen(path, values)
    if text_type == QWEN:
        raise ValueError("native Qwen RL requires a flat qwen3_moe config")
    for where, model_type in (("model_type", root_type), ("text_config.model_type", text_type)):
        if model_type not in DSV4_TYPES:
            raise ValueError(f"unsupported {where}: {model_type!r}")
    return _load_deepseek(path, values, text)


def _check_policy_request(model_config, random_init, trainable_scope, lora_config, initial_adapter, sft_source):
    if sft_source is not None and (random_init or trainable_scope != "all" or is_qwen(model_config)):
        raise ValueError("an SFT source requires a pretrained DSV4 base and trainable_scope=all")
    if (lora_config is not None) != (trainable_scope == "lora"):
        raise ValueError("LoRA scope requires an explicit adapter configuration")
    if initial_adapter is not None and lora_config is None:
        raise ValueError("initial_adapter requires LoRA")
    if lora_config is not None and lora_config.dropout != 0:
        raise ValueError("LoRA RL requires dropout=0")
    if not is_qwen(model_config) and trainable_scope not in ("all", "lora"):
        raise ValueError("DeepSeek RL requires trainable_scope=all or lora")


def build_policy(model_dir, model_config, *, random_init, devices, dtype, trainable_scope="all", lora_config=None,
                 initial_adapter=None, engram_offload=True, sft_source=None):
    _check_policy_request(model_config, random_init, trainable_scope, lora_config, initial_adapter, sft_source)
    common = dict(random_init=random_init, devices=devices, dtype=dtype, lora_config=lora_config,
                  initial_adapter=initial_adapter)
    if is_qwen(model_config):
        model = build_qwen_policy(model_dir, model_config, trainable_scope=trainable_scope, **common)
    else:
        model = build_dsv41_policy(model_dir, model_config, engram_offload=engram_offload, sft_source=sft_source,
                                   **common)
    if lora_config is not None:
        model.lora_metadata = lora_metadata(lora_config, initial_adapter)
    return model


__all__ = ["build_policy", "initial_sft_source", "is_qwen", "load_model_config", "policy_lora_config"]
