"""RL prompt data and the reward functions that score sampled responses.

Input format (one JSON object per line, the interface of ``dsv41_train/rl/data.py``): exactly one
prompt field - ``prompt_ids`` (token ids), ``prompt`` (text) or ``messages`` (chat turns), the
last two encoded by the checkpoint's tokenizer - plus optional ``target_ids`` and ``metadata``;
every other key is folded into the metadata.

Reward specs resolve in this order: a text reward of :mod:`.rewards` (needs the tokenizer), a
built-in token reward (``token_accuracy``, ``exact_match``, ``toy_token_score``), or a plugin
``module:function``. Every resolved reward is wrapped so that a non-finite score is an error.
"""

from __future__ import annotations

import importlib
import json
import math
import warnings
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Callable, Mapping, Optional

PROMPT_FIELDS = ("prompt_ids", "prompt", "messages")
_RESERVED = frozenset({"prompt_ids", "target_ids", "metadata"})


def validate_token_ids(value: Any, name: str, *, allow_empty: bool = False) -> list[int]:
    """``value`` as a list of token ids (plain ints >= 0; bools are not ids)."""
    if not isinstance(value, (list, tuple)):
        raise ValueError(f"{name} must be a list of nonnegative integer token IDs")
    ids = list(value)
    if not ids and not allow_empty:
        raise ValueError(f"{name} must not be empty")
    if not all(_is_token(t) for t in ids):
        raise ValueError(f"{name} must contain only nonnegative integer token IDs")
    return ids


def _is_token(value: Any) -> bool:
    return isinstance(value, int) and not isinstance(value, bool) and value >= 0


def _as_metadata(value: Any) -> dict[str, Any]:
    if not isinstance(value, dict):
        raise ValueError("metadata must be a JSON object")
    return dict(value)


@dataclass
class PromptRecord:
    prompt_ids: list[int]
    target_ids: Optional[list[int]] = None
    metadata: dict[str, Any] = field(default_factory=dict)

    def __post_init__(self) -> None:
        self.prompt_ids = validate_token_ids(self.prompt_ids, "prompt_ids")
        if self.target_ids is not None:
            self.target_ids = validate_token_ids(self.target_ids, "target_ids", allow_empty=True)
        self.metadata = _as_metadata(self.metadata)

    @classmethod
    def from_mapping(cls, value: Mapping[str, Any], *, tokenizer=None) -> "PromptRecord":
        if not isinstance(value, Mapping):
            raise ValueError("each JSONL record must be an object")
        present = [name for name in PROMPT_FIELDS if name in value]
        if len(present) != 1:
            raise ValueError("each JSONL record requires exactly one of prompt_ids, prompt or messages")
        if present[0] == "prompt_ids":
            prompt_ids = value["prompt_ids"]
        elif tokenizer is None:
            raise ValueError("text records require tokenizer.json in the model directory")
        else:
            prompt_ids = tokenizer.encode_prompt(prompt=value.get("prompt"), messages=value.get("messages"))
        metadata = _as_metadata(value.get("metadata", {}))
        for key, item in value.items():
            if key not in _RESERVED:
                metadata[key] = item
        return cls(prompt_ids, value.get("target_ids"), metadata)


RewardFn = Callable[[PromptRecord, list[int]], float]


def _read_records(path, tokenizer):
    """(line number, record) for every non-blank line; errors carry the line."""
    with Path(path).open(encoding="utf-8") as stream:
        for number, line in enumerate(stream, 1):
            if line.strip():
                try:
                    yield number, PromptRecord.from_mapping(json.loads(line), tokenizer=tokenizer)
                except (ValueError, TypeError) as exc:
                    raise ValueError(f"{path}:{number}: {exc}") from exc


def load_jsonl(path, *, tokenizer=None, max_prompt_tokens=None, length_policy="error") -> list[PromptRecord]:
    """Records of a JSONL file. Prompts longer than ``max_prompt_tokens`` raise
    (``length_policy="error"``) or are dropped with one warning (``"skip"``)."""
    if length_policy not in ("error", "skip"):
        raise ValueError("length_policy must be error or skip")
    kept: list[PromptRecord] = []
    dropped = 0
    for number, record in _read_records(path, tokenizer):
        length = len(record.prompt_ids)
        if max_prompt_tokens is None or length <= max_prompt_tokens:
            kept.append(record)
        elif length_policy == "skip":
            dropped += 1
        else:
            raise ValueError(f"{path}:{number}: prompt length {length} exceeds limit {max_prompt_tokens}")
    if dropped:
        warnings.warn(f"{path}: skipped {dropped} records exceeding the prompt length limit", stacklevel=2)
    if not kept:
        raise ValueError(f"{path}: no records found")
    return kept


# -- built-in token rewards ---------------------------------------------------------------------
def _require_target(record: PromptRecord) -> list[int]:
    if record.target_ids is None:
        raise ValueError("this reward requires target_ids in every JSONL record")
    return record.target_ids


def token_accuracy(record: PromptRecord, response_ids: list[int]) -> float:
    """Position-wise matches with the target over the longer of the two sequences."""
    target = _require_target(record)
    longest = max(len(target), len(response_ids))
    if longest == 0:
        return 1.0
    return sum(1 for a, b in zip(target, response_ids) if a == b) / longest


def exact_match(record: PromptRecord, response_ids: list[int]) -> float:
    return 1.0 if list(response_ids) == _require_target(record) else 0.0


def toy_token_score(record: PromptRecord, response_ids: list[int]) -> float:
    """Mean token id of the response (a smoke-test reward)."""
    if not response_ids:
        raise ValueError("toy_token_score requires at least one response token")
    return sum(response_ids) / len(response_ids)


BUILTIN_REWARDS: dict[str, RewardFn] = {
    "token_accuracy": token_accuracy, "exact_match": exact_match, "toy_token_score": toy_token_score,
}


def _plugin(spec: str) -> Callable:
    module_name, colon, attribute = spec.partition(":")
    if not (colon and module_name and attribute) or ":" in attribute:
        raise ValueError(f"unknown reward {spec!r}; use a builtin or module:function")
    target = getattr(importlib.import_module(module_name), attribute)
    if not callable(target):
        raise ValueError(f"reward {spec!r} is not callable")
    return target


def build_reward(spec: str, *, tokenizer=None) -> RewardFn:
    """The reward named by ``spec``; the returned callable raises on non-finite scores and carries
    ``strip_stop_tokens`` (true for text rewards, which score the text without stop tokens)."""
    from .rewards import TEXT_REWARDS, build_text_reward

    text = spec in TEXT_REWARDS
    if text:
        if tokenizer is None:
            raise ValueError(f"reward {spec!r} requires tokenizer.json in the model directory")
        scorer = build_text_reward(spec, tokenizer)
    else:
        scorer = BUILTIN_REWARDS.get(spec) or _plugin(spec)

    def reward(record: PromptRecord, response_ids: list[int]) -> float:
        value = float(scorer(record, response_ids))
        if math.isfinite(value):
            return value
        raise ValueError(f"reward {spec!r} returned a non-finite value")

    reward.strip_stop_tokens = text
    return reward


__all__ = ["BUILTIN_REWARDS", "PromptRecord", "RewardFn", "build_reward", "exact_match", "load_jsonl",
           "token_accuracy", "toy_token_score", "validate_token_ids"]
