"""Native autoregressive sampling of GRPO groups, recording the behaviour log-probability of every
sampled action.

Sampling semantics follow ``dsv41_train/rl/rollout.py`` (the learner's importance ratios are
computed against these numbers): categorical sampling at temperature T from a CPU generator; a
response ends at the longest matching stop sequence ("stop") or an EOS id ("eos"), both kept in
the response with their log-probabilities, or at ``max_new_tokens`` ("length"); text rewards
score the response without its stop tokens; ``truncated_reward`` (if set) replaces the reward of a
length-truncated sample while ``raw_reward`` keeps the scored value. A model with a
``next_token_logits`` hook (the Qwen KV cache) is stepped through it.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional, Sequence

import torch
from torch import nn

from .algorithm import input_device, validate_temperature
from .data import PromptRecord, RewardFn, build_reward, validate_token_ids

FINISH_REASONS = ("eos", "stop", "length")


def _positive_int(value, name: str) -> int:
    if isinstance(value, bool) or not isinstance(value, int) or value <= 0:
        raise ValueError(f"{name} must be a positive integer")
    return value


@dataclass
class Sample:
    prompt_ids: list[int]
    response_ids: list[int]
    behavior_log_probs: list[float]
    reward: float
    policy_version: int
    finish_reason: str = "length"
    stop_token_count: int = 0
    raw_reward: Optional[float] = None

    def __post_init__(self) -> None:
        self.prompt_ids = validate_token_ids(self.prompt_ids, "prompt_ids")
        self.response_ids = validate_token_ids(self.response_ids, "response_ids")
        self.behavior_log_probs = list(map(float, self.behavior_log_probs))
        if len(self.behavior_log_probs) != len(self.response_ids):
            raise ValueError("each response token requires one behavior log probability")
        if not all(math.isfinite(v) and v <= 1e-6 for v in self.behavior_log_probs):
            raise ValueError("behavior log probabilities must be finite and nonpositive")
        self.reward = float(self.reward)
        if not math.isfinite(self.reward):
            raise ValueError("reward must be finite")
        self.raw_reward = float(self.reward if self.raw_reward is None else self.raw_reward)
        if self.finish_reason not in FINISH_REASONS:
            raise ValueError("finish_reason must be eos, stop or length")
        count = self.stop_token_count
        if type(count) is not int or not 0 <= count <= len(self.response_ids):
            raise ValueError("invalid stop_token_count")
        version = self.policy_version
        if isinstance(version, bool) or not isinstance(version, int) or version < 0:
            raise ValueError("policy_version must be a nonnegative integer")

    @property
    def content_ids(self):
        """The response without its trailing stop / EOS tokens."""
        return self.response_ids[:len(self.response_ids) - self.stop_token_count]


@dataclass
class RolloutGroup:
    samples: list[Sample]
    group_id: int
    policy_version: int

    def __post_init__(self) -> None:
        if not self.samples:
            raise ValueError("a rollout group must not be empty")
        if any(s.policy_version != self.policy_version for s in self.samples):
            raise ValueError("all group samples must have the group policy_version")
        prompt = self.samples[0].prompt_ids
        if any(s.prompt_ids != prompt for s in self.samples[1:]):
            raise ValueError("all group samples must have the same prompt")


class _Terminator:
    """Decides after every sampled token whether the response has ended."""

    def __init__(self, eos_token_id, stop_token_sequences) -> None:
        if eos_token_id is None:
            self.eos = frozenset()
        else:
            ids = [eos_token_id] if isinstance(eos_token_id, int) else list(eos_token_id)
            self.eos = frozenset(validate_token_ids(ids, "eos_token_id", allow_empty=True))
        stops = [validate_token_ids(list(seq), "stop_token_sequences") for seq in stop_token_sequences]
        self.stops = sorted(stops, key=len, reverse=True)  # the longest match wins

    def __call__(self, response: list[int]) -> tuple[str, int] | None:
        for seq in self.stops:
            if len(response) >= len(seq) and response[-len(seq):] == seq:
                return "stop", len(seq)
        return ("eos", 1) if response[-1] in self.eos else None


def _next_logits(model, tokens: torch.Tensor) -> torch.Tensor:
    mask = torch.ones_like(tokens)
    hook = getattr(model, "next_token_logits", None)
    if hook is not None:
        return hook(tokens, attention_mask=mask)[0]
    out = model(tokens, attention_mask=mask)
    logits = out if isinstance(out, torch.Tensor) else out.logits
    if logits.ndim != 3 or logits.shape[1] != tokens.shape[1]:
        raise ValueError("model must return one logits vector per input token")
    return logits[0, -1]


def _sample_response(model, prompt, max_new_tokens, temperature, terminator, generator, device):
    response, log_probs = [], []
    for _ in range(max_new_tokens):
        context = torch.tensor([prompt + response], dtype=torch.long, device=device)
        distribution = torch.log_softmax(_next_logits(model, context).float() / temperature, dim=-1)
        if not bool(torch.isfinite(distribution).all()):
            raise ValueError("generation log probabilities contain non-finite values")
        token = int(torch.multinomial(distribution.exp().cpu(), 1, generator=generator))
        response.append(token)
        log_probs.append(float(distribution[token]))
        ended = terminator(response)
        if ended is not None:
            return response, log_probs, ended
    return response, log_probs, ("length", 0)


def generate_group(model: nn.Module, record, group_size: int, max_new_tokens: int, temperature: float,
                   eos_token_id, policy_version: int, group_id: int, generator: Optional[torch.Generator] = None,
                   reward_fn: Optional[RewardFn] = None, stop_token_sequences: Sequence[Sequence[int]] = (),
                   truncated_reward: Optional[float] = None) -> RolloutGroup:
    validate_temperature(temperature)
    _positive_int(group_size, "group_size")
    _positive_int(max_new_tokens, "max_new_tokens")
    terminator = _Terminator(eos_token_id, stop_token_sequences)
    if generator is not None and generator.device.type != "cpu":
        raise ValueError("generation requires a CPU torch.Generator")
    record = record if isinstance(record, PromptRecord) else PromptRecord.from_mapping(record)
    reward_fn = reward_fn or build_reward("token_accuracy")
    strip = getattr(reward_fn, "strip_stop_tokens", False)
    device = input_device(model)
    samples = []
    training = model.training
    model.eval()
    try:
        with torch.inference_mode():
            for _ in range(group_size):
                response, log_probs, (finish, stops) = _sample_response(
                    model, record.prompt_ids, max_new_tokens, temperature, terminator, generator, device)
                scored = response[:len(response) - stops] if strip else response
                raw = float(reward_fn(record, scored))
                reward = truncated_reward if (finish == "length" and truncated_reward is not None) else raw
                samples.append(Sample(record.prompt_ids, response, log_probs, reward, policy_version, finish, stops, raw))
    finally:
        model.train(training)
    return RolloutGroup(samples, group_id, policy_version)


def generation_options(model_dir, model_config, config) -> dict:
    """EOS ids (the run config's, or the checkpoint's generation config), stop sequences and the
    truncation reward, with every id checked against the vocabulary."""
    from .tokenizer import read_eos_token_ids

    eos = (tuple(config.eos_token_ids) if config.eos_token_ids is not None
           else read_eos_token_ids(model_dir, model_config.eos_token_id))
    every_id = [*eos, *(t for seq in config.stop_token_sequences for t in seq)]
    if any(t >= model_config.vocab_size for t in every_id):
        raise ValueError("stop token ID is outside the model vocabulary")
    return {"eos_token_id": eos, "stop_token_sequences": config.stop_token_sequences,
            "truncated_reward": config.truncated_reward}


__all__ = ["RolloutGroup", "Sample", "generate_group", "generation_options"]
