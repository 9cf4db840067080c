"""Model-family selection for the RL runtime (``dsv41_train/rl/family.py:11-99``).

``config.json`` with ``model_type == "qwen3_moe"`` (flat, unquantized) selects Qwen3-MoE;
``deepseek_v41`` / ``deepseek_v41_text`` or no type selects DeepSeek-V4.1.
"""

from __future__ import annotations

import json
from dataclasses import asdict
from pathlib import Path

from ..lora import LoRAConfig
from .policy import build_dsv41_policy, build_qwen_policy, validate_qwen_config

QWEN_LORA_TARGETS = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj")


def policy_lora_config(config, model_config):
    if config.trainable_scope != "lora":
        return None
    targets = config.lora_targets
    if targets is None:
        targets = QWEN_LORA_TARGETS if getattr(model_config, "model_type", None) == "qwen3_moe" else LoRAConfig().targets
    return LoRAConfig(config.lora_rank, config.lora_alpha, config.lora_dropout, targets)


def lora_metadata(lora_config, initial_adapter) -> dict:
    from .checkpoint import file_sha256

    return json.loads(json.dumps({"config": asdict(lora_config),
                                  "initial_adapter_sha256": file_sha256(initial_adapter) if initial_adapter else None}))


def initial_sft_source(model_dir, model_config, config, random_init):
    """The full-SFT snapshot named by ``initial_sft_checkpoint`` (DSV4 with pretrained base only)."""
    if config.initial_sft_checkpoint is None:
        return None
    if random_init or getattr(model_config, "model_type", None) == "qwen3_moe":
        raise ValueError("initial_sft_checkpoint requires a pretrained DSV4 base")
    from ..train.sft_source import SFTCheckpointSource

    return SFTCheckpointSource(config.initial_sft_checkpoint, model_dir)


def load_model_config(model_dir):
    path = Path(model_dir) / "config.json"
    values = json.loads(path.read_text(encoding="utf-8"))
    if not isinstance(values, dict):
        raise ValueError("model config must be an object")
    text = values.get("text_config")
    if text is not None and not isinstance(text, dict):
        raise ValueError("text_config must be an object")
    root_type, text_type = values.get("model_type"), (text or {}).get("model_type")
    if root_type == "qwen3_moe":
        if text is not None:
            raise ValueError("native Qwen RL requires a flat qwen3_moe config")
        if values.get("quantization_config"):
            raise ValueError("native Qwen RL requires unquantized mounted safetensors")
        from ..models.qwen import Qwen3MoeConfig

        config = Qwen3MoeConfig.from_json(path)
        validate_qwen_config(config)
        return config
    if text_type == "qwen3_moe":
        raise ValueError("native Qwen RL requires a flat qwen3_moe config")
    for name, model_type in (("model_type", root_type), ("text_config.model_type", text_type)):
        if model_type not in (None, "deepseek_v41", "deepseek_v41_text"):
            raise ValueError(f"unsupported {name}: {model_type!r}")
    from ..models.dsv4.config import DeepSeekV41Config

    config = DeepSeekV41Config.from_json(path)
    quantized = bool(values.get("quantization_config") or (text or {}).get("quantization_config"))
    config.checkpoint_format = values.get("checkpoint_format", "released" if quantized else "native")
    if config.checkpoint_format == "tiny_dsv41":
        config.checkpoint_format = "native"
    if config.checkpoint_format not in {"native", "released"}:
        raise ValueError("DeepSeek checkpoint_format must be native or released")
    if config.attention_dropout:
        raise ValueError("RL policies require attention_dropout=0 for behavior probability consistency")
    return config


def build_policy(model_dir, model_config, *, random_init, devices, dtype, trainable_scope="all", lora_config=None,
                 initial_adapter=None, engram_offload=True, sft_source=None):
    if sft_source is not None and (random_init or trainable_scope != "all"
                                   or getattr(model_config, "model_type", None) == "qwen3_moe"):
        raise ValueError("an SFT source requires a pretrained DSV4 base and trainable_scope=all")
    if (trainable_scope == "lora") != (lora_config is not None):
        raise ValueError("LoRA scope requires an explicit adapter configuration")
    if initial_adapter is not None and lora_config is None:
        raise ValueError("initial_adapter requires LoRA")
    if lora_config is not None and lora_config.dropout != 0:
        raise ValueError("LoRA RL requires dropout=0")
    if getattr(model_config, "model_type", None) == "qwen3_moe":
        model = build_qwen_policy(model_dir, model_config, random_init=random_init, devices=devices, dtype=dtype,
                                  trainable_scope=trainable_scope, lora_config=lora_config,
                                  initial_adapter=initial_adapter)
    else:
        if trainable_scope not in {"all", "lora"}:
            raise ValueError("DeepSeek RL requires trainable_scope=all or lora")
        model = build_dsv41_policy(model_dir, model_config, random_init=random_init, devices=devices, dtype=dtype,
                                   lora_config=lora_config, initial_adapter=initial_adapter,
                                   engram_offload=engram_offload, sft_source=sft_source)
    if lora_config is not None:
        model.lora_metadata = lora_metadata(lora_config, initial_adapter)
    return model


__all__ = ["build_policy", "load_model_config", "policy_lora_config"]
