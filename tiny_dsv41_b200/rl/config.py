"""RL run configuration.

The field names, defaults and JSON form are the interface of ``dsv41_train/rl/config.py`` (a run
directory written by either side loads on the other). Validation is table driven here: per-field
kind checks (``_FIELD_RULES``) and cross-field requirements (``_REQUIREMENTS``), each a predicate
plus the message of the error it raises.

``trainer_num_gpus`` / ``rollout_num_gpus`` in a JSON file expand into explicit device lists:
learner GPUs ``cuda:0 .. cuda:T-1``, then rollout GPUs ``cuda:T .. cuda:T+R-1``; a count of zero
selects the CPU.
"""

from __future__ import annotations

import json
import math
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Any, Callable


@dataclass(frozen=True)
class RLConfig:
    max_steps: int = 3
    group_size: int = 4
    groups_per_step: int = 1
    max_new_tokens: int = 4
    temperature: float = 1.0
    clip_eps: float = 0.2
    kl_beta: float = 0.0
    learning_rate: float = 1e-4
    weight_decay: float = 0.0
    max_grad_norm: float = 1.0
    max_policy_lag: int = 2
    queue_capacity: int = 2
    reward: str = "token_accuracy"
    learner_devices: tuple[str, ...] = ("cpu",)
    rollout_devices: tuple[str, ...] = ("cpu",)
    rollout_engine: str = "vllm"
    engram_offload: bool = True
    train_engram: bool = False
    engram_cache_mib: int = 0
    optimizer: str = "adamw"
    initial_engram_delta: str | None = None
    initial_sft_checkpoint: str | None = None
    trainable_scope: str = "all"
    lora_rank: int = 8
    lora_alpha: float = 16.0
    lora_dropout: float = 0.0
    lora_targets: tuple[str, ...] | None = None
    initial_adapter: str | None = None
    qwen_last_position_only: bool = False
    qwen_kv_cache: bool = False
    backprop_chunk_tokens: int = 0
    gradient_checkpointing: bool = False
    dtype: str = "float32"
    seed: int = 42
    num_threads: int = 1
    checkpoint_interval: int = 1
    output_dir: str = "runs/default"
    worker_timeout_seconds: float = 600.0
    max_prompt_tokens: int | None = None
    length_policy: str = "error"
    eos_token_ids: tuple[int, ...] | None = None
    stop_token_sequences: tuple[tuple[int, ...], ...] = ()
    truncated_reward: float | None = None
    eval_interval: int = 0
    eval_samples_per_prompt: int = 1
    eval_seed: int = 1234
    log_samples_per_step: int = 1

    @classmethod
    def from_dict(cls, values: dict) -> "RLConfig":
        config = cls(**_normalise(dict(values)))
        config.validate()
        return config

    @classmethod
    def from_json(cls, path) -> "RLConfig":
        return cls.from_dict(json.loads(Path(path).read_text(encoding="utf-8")))

    def to_dict(self) -> dict:
        return asdict(self)

    def validate(self) -> None:
        for names, ok, message in _FIELD_RULES:
            for name in names:
                if not ok(getattr(self, name)):
                    raise ValueError(message.format(name=name))
        for ok, message in _REQUIREMENTS:
            if not ok(self):
                raise ValueError(message)
        if self.trainable_scope == "lora":
            from ..lora import LoRAConfig

            # constructing the adapter config applies its own rank / alpha / dropout / target rules
            LoRAConfig(self.lora_rank, self.lora_alpha, self.lora_dropout,
                       LoRAConfig().targets if self.lora_targets is None else self.lora_targets)


# -- JSON normalisation ---------------------------------------------------------------------------
def _devices_from_counts(values: dict) -> None:
    trainer, rollout = values.pop("trainer_num_gpus"), values.pop("rollout_num_gpus")
    if not all(type(n) is int and n >= 0 for n in (trainer, rollout)):
        raise ValueError("GPU counts must be nonnegative integers; zero selects CPU")
    values["learner_devices"] = tuple(f"cuda:{i}" for i in range(trainer)) or ("cpu",)
    values["rollout_devices"] = tuple(f"cuda:{trainer + i}" for i in range(rollout)) or ("cpu",)


def _normalise(values: dict) -> dict:
    counts = [n in values for n in ("trainer_num_gpus", "rollout_num_gpus")]
    if any(counts):
        if not all(counts):
            raise ValueError("specify both trainer_num_gpus and rollout_num_gpus")
        if "learner_devices" in values or "rollout_devices" in values:
            raise ValueError("specify GPU counts or explicit device lists, not both")
        _devices_from_counts(values)
    # JSON arrays become the tuples the frozen dataclass holds
    for name in ("learner_devices", "rollout_devices", "lora_targets", "eos_token_ids"):
        if values.get(name) is not None:
            values[name] = tuple(values[name])
    if "stop_token_sequences" in values:
        values["stop_token_sequences"] = tuple(tuple(seq) for seq in values["stop_token_sequences"])
    return values


# -- per-field rules --------------------------------------------------------------------------------
def _int(value) -> bool:
    return type(value) is int


def _token(value) -> bool:
    return _int(value) and value >= 0


def _finite(value) -> bool:
    return isinstance(value, (int, float)) and math.isfinite(value)


def _device_list(devices) -> bool:
    if not devices or len(set(devices)) != len(devices):
        return False
    return devices == ("cpu",) or all(isinstance(d, str) and d.startswith("cuda:") and d[5:].isdigit()
                                      for d in devices)


_U63 = 2 ** 63 - 1
_FIELD_RULES: list[tuple[tuple[str, ...], Callable[[Any], bool], str]] = [
    (("rollout_engine",), lambda v: v in ("vllm", "native-pytorch"), "rollout_engine must be vllm or native-pytorch"),
    (("max_steps", "groups_per_step", "max_new_tokens", "queue_capacity", "num_threads", "checkpoint_interval",
      "eval_samples_per_prompt"), lambda v: _int(v) and v >= 1, "{name} must be a positive integer"),
    (("group_size",), lambda v: _int(v) and v >= 2, "group_size must be at least two"),
    (("max_policy_lag",), _token, "max_policy_lag must be a nonnegative integer"),
    (("eval_interval", "log_samples_per_step", "eval_seed", "seed"), lambda v: _int(v) and 0 <= v < _U63,
     "{name} must be a nonnegative integer below 2**63 - 1"),
    (("max_prompt_tokens",), lambda v: v is None or (_int(v) and v >= 1),
     "max_prompt_tokens must be a positive integer or null"),
    (("length_policy",), lambda v: v in ("error", "skip"), "length_policy must be error or skip"),
    (("eos_token_ids",), lambda v: v is None or all(map(_token, v)),
     "eos_token_ids must contain nonnegative integer IDs or be null"),
    (("stop_token_sequences",), lambda v: all(seq and all(map(_token, seq)) for seq in v),
     "stop_token_sequences must contain nonempty lists of nonnegative integer IDs"),
    (("truncated_reward",), lambda v: v is None or _finite(v), "truncated_reward must be finite or null"),
    (("temperature", "learning_rate", "max_grad_norm", "worker_timeout_seconds"), lambda v: _finite(v) and v > 0,
     "{name} must be finite and positive"),
    (("kl_beta", "weight_decay"), lambda v: _finite(v) and v >= 0, "{name} must be finite and nonnegative"),
    (("clip_eps",), lambda v: _finite(v) and 0 < v < 1, "clip_eps must be in (0, 1)"),
    (("dtype",), lambda v: v in ("float32", "bfloat16"), "dtype must be float32 or bfloat16"),
    (("trainable_scope",), lambda v: v in ("all", "lm_head", "lora"), "trainable_scope must be all, lm_head or lora"),
    (("optimizer",), lambda v: v in ("adamw", "sgd"), "optimizer must be adamw or sgd"),
    (("engram_cache_mib", "backprop_chunk_tokens"), _token, "{name} must be a nonnegative integer"),
    (("reward", "output_dir"), bool, "reward and output_dir must not be empty"),
    (("learner_devices", "rollout_devices"), _device_list,
     "device lists must be nonempty with no duplicates: use ['cpu'] or explicit CUDA devices such as "
     "['cuda:0', 'cuda:1']"),
]


# -- cross-field requirements ---------------------------------------------------------------------
def _native(c: RLConfig) -> bool:
    return c.rollout_engine == "native-pytorch"


_REQUIREMENTS: list[tuple[Callable[[RLConfig], bool], str]] = [
    (lambda c: not c.train_engram or (c.engram_offload and _native(c) and c.optimizer == "sgd"
                                      and c.weight_decay == 0 and c.trainable_scope in ("all", "lora")),
     "train_engram requires Engram offload, native-pytorch, SGD with zero weight decay and trainable_scope=all "
     "or lora"),
    (lambda c: not c.engram_cache_mib or c.engram_offload, "engram_cache_mib requires Engram offload"),
    (lambda c: c.initial_engram_delta is None or (c.engram_offload and _native(c)),
     "initial_engram_delta requires Engram offload and native-pytorch"),
    (lambda c: c.initial_sft_checkpoint is None or (_native(c) and c.trainable_scope == "all" and c.engram_offload
                                                    and c.initial_adapter is None and c.initial_engram_delta is None),
     "initial_sft_checkpoint requires native-pytorch, trainable_scope=all, CPU Engram offload and no initial "
     "adapter or Engram delta"),
    (lambda c: c.trainable_scope != "lora" or (_native(c) and c.lora_dropout == 0),
     "Local-manager LoRA RL requires native-pytorch and lora_dropout=0"),
    (lambda c: c.trainable_scope == "lora" or c.initial_adapter is None, "initial_adapter requires trainable_scope=lora"),
    (lambda c: not c.qwen_kv_cache or (c.trainable_scope == "lm_head" and c.qwen_last_position_only
                                       and not c.backprop_chunk_tokens),
     "qwen_kv_cache requires lm_head, last-position logits and unchunked turn replay"),
]


__all__ = ["RLConfig"]
