"""Prompt records (token ids or text through the checkpoint tokenizer) and built-in rewards.

``PromptRecord``, ``load_jsonl``, ``token_accuracy``, ``exact_match``, ``toy_token_score`` and
``build_reward`` (builtin name, text reward, or ``module:function`` plugin) with the behaviour of
``dsv41_train/rl/data.py``.
"""

from __future__ import annotations

import importlib
import json
import math
import warnings
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Callable, Mapping, Optional


def validate_token_ids(value: Any, name: str, *, allow_empty: bool = False) -> list[int]:
    if not isinstance(value, (list, tuple)):
        raise ValueError(f"{name} must be a list of nonnegative integer token IDs")
    if not value and not allow_empty:
        raise ValueError(f"{name} must not be empty")
    if any(isinstance(t, bool) or not isinstance(t, int) or t < 0 for t in value):
        raise ValueError(f"{name} must contain only nonnegative integer token IDs")
    return list(value)


@dataclass
class PromptRecord:
    prompt_ids: list[int]
    target_ids: Optional[list[int]] = None
    metadata: dict[str, Any] = field(default_factory=dict)

    def __post_init__(self) -> None:
        self.prompt_ids = validate_token_ids(self.prompt_ids, "prompt_ids")
        if self.target_ids is not None:
            self.target_ids = validate_token_ids(self.target_ids, "target_ids", allow_empty=True)
        if not isinstance(self.metadata, dict):
            raise ValueError("metadata must be a JSON object")
        self.metadata = dict(self.metadata)

    @classmethod
    def from_mapping(cls, value: Mapping[str, Any], *, tokenizer=None) -> "PromptRecord":
        if not isinstance(value, Mapping):
            raise ValueError("each JSONL record must be an object")
        if sum(n in value for n in ("prompt_ids", "prompt", "messages")) != 1:
            raise ValueError("each JSONL record requires exactly one of prompt_ids, prompt or messages")
        prompt_ids = value.get("prompt_ids")
        if "prompt_ids" not in value:
            if tokenizer is None:
                raise ValueError("text records require tokenizer.json in the model directory")
            prompt_ids = tokenizer.encode_prompt(prompt=value.get("prompt"), messages=value.get("messages"))
        metadata = value.get("metadata", {})
        if not isinstance(metadata, dict):
            raise ValueError("metadata must be a JSON object")
        metadata = dict(metadata)
        metadata.update({k: v for k, v in value.items() if k not in {"prompt_ids", "target_ids", "metadata"}})
        return cls(prompt_ids, value.get("target_ids"), metadata)


RewardFn = Callable[[PromptRecord, list[int]], float]


def load_jsonl(path, *, tokenizer=None, max_prompt_tokens=None, length_policy="error") -> list[PromptRecord]:
    if length_policy not in {"error", "skip"}:
        raise ValueError("length_policy must be error or skip")
    records, skipped = [], 0
    with Path(path).open(encoding="utf-8") as stream:
        for number, line in enumerate(stream, 1):
            if not line.strip():
                continue
            try:
                record = PromptRecord.from_mapping(json.loads(line), tokenizer=tokenizer)
                if max_prompt_tokens is not None and len(record.prompt_ids) > max_prompt_tokens:
                    if length_policy == "skip":
                        skipped += 1
                        continue
                    raise ValueError(f"prompt length {len(record.prompt_ids)} exceeds limit {max_prompt_tokens}")
                records.append(record)
            except (ValueError, TypeError) as exc:
                raise ValueError(f"{path}:{number}: {exc}") from exc
    if skipped:
        warnings.warn(f"{path}: skipped {skipped} records exceeding the prompt length limit", stacklevel=2)
    if not records:
        raise ValueError(f"{path}: no records found")
    return records


def _target(record: PromptRecord) -> list[int]:
    if record.target_ids is None:
        raise ValueError("this reward requires target_ids in every JSONL record")
    return record.target_ids


def token_accuracy(record: PromptRecord, response_ids: list[int]) -> float:
    target = _target(record)
    denominator = max(len(target), len(response_ids))
    return 1.0 if denominator == 0 else sum(a == b for a, b in zip(target, response_ids)) / denominator


def exact_match(record: PromptRecord, response_ids: list[int]) -> float:
    return float(response_ids == _target(record))


def toy_token_score(record: PromptRecord, response_ids: list[int]) -> float:
    if not response_ids:
        raise ValueError("toy_token_score requires at least one response token")
    return sum(response_ids) / len(response_ids)


def build_reward(spec: str, *, tokenizer=None) -> RewardFn:
    builtins = {"token_accuracy": token_accuracy, "exact_match": exact_match, "toy_token_score": toy_token_score}
    from .rewards import TEXT_REWARDS, build_text_reward

    if spec in TEXT_REWARDS:
        if tokenizer is None:
            raise ValueError(f"reward {spec!r} requires tokenizer.json in the model directory")
        fn = build_text_reward(spec, tokenizer)
    elif spec in builtins:
        fn = builtins[spec]
    else:
        module_name, sep, function_name = spec.partition(":")
        if not sep or not module_name or not function_name or ":" in function_name:
            raise ValueError(f"unknown reward {spec!r}; use a builtin or module:function")
        fn = getattr(importlib.import_module(module_name), function_name)
        if not callable(fn):
            raise ValueError(f"reward {spec!r} is not callable")

    def checked(record: PromptRecord, response_ids: list[int]) -> float:
        reward = float(fn(record, response_ids))
        if not math.isfinite(reward):
            raise ValueError(f"reward {spec!r} returned a non-finite value")
        return reward

    checked.strip_stop_tokens = spec in TEXT_REWARDS
    return checked


__all__ = ["PromptRecord", "RewardFn", "build_reward", "exact_match", "load_jsonl", "token_accuracy",
           "toy_token_score", "validate_token_ids"]
