"""Prompt-response backend: one GRPO sample of a prompt with this library's policy
(the native sampler behind ``rollout_manager/backends/pytorch_rl.py:15-179``).

The plan payload carries ``{"prompt_response": {"record": {prompt_ids, target_ids, metadata},
"group_id": ..., "policy": {version, ...}}}``; the backend samples with a CPU generator seeded by
the episode's ``sampling_seed`` and reports the response, behaviour log-probs and reward as the
episode's native outcome. Sampling runs in a worker thread so the event loop stays responsive;
a cancelled episode returns without a score.
"""

from __future__ import annotations

import asyncio

import torch

from ..rl.data import PromptRecord
from ..rl.rollout import generate_group
from .contracts import EpisodePlan, EpisodeResult


class PromptResponseBackend:
    def __init__(self, model, reward_fn, *, max_new_tokens: int, temperature: float, eos_token_id=(),
                 stop_token_sequences=(), policy_version: int = 0) -> None:
        self.model, self.reward_fn = model, reward_fn
        self.max_new_tokens, self.temperature = max_new_tokens, temperature
        self.eos, self.stops = eos_token_id, stop_token_sequences
        self.policy_version = policy_version
        self._lock = asyncio.Lock()

    def _sample(self, plan: EpisodePlan):
        payload = plan.task.payload["prompt_response"]
        record = PromptRecord(**payload["record"])
        seed = plan.identity.sampling_seed if plan.identity.sampling_seed is not None else plan.identity.sample_index
        gen = torch.Generator().manual_seed(seed)
        group = generate_group(self.model, record, 1, self.max_new_tokens, self.temperature, self.eos,
                               self.policy_version, int(payload.get("group_id", 0)), gen, self.reward_fn,
                               self.stops)
        return group.samples[0]

    async def execute(self, plan: EpisodePlan, cancellation) -> EpisodeResult:
        if cancellation.cancelled():
            return EpisodeResult(plan.identity, "cancelled", "not_verified", False, "clean",
                                 {"reason": cancellation.reason}, None)
        async with self._lock:  # one model, one sampler at a time
            sample = await asyncio.to_thread(self._sample, plan)
        outcome = {"response_ids": sample.response_ids, "behavior_log_probs": sample.behavior_log_probs,
                   "reward": sample.reward, "raw_reward": sample.raw_reward, "finish_reason": sample.finish_reason,
                   "stop_token_count": sample.stop_token_count, "policy_version": sample.policy_version}
        return EpisodeResult(plan.identity, "completed", "verified", True, "clean", outcome, None,
                             usage={"output_tokens": len(sample.response_ids)},
                             source_sha256=plan.task.source_sha256)


__all__ = ["PromptResponseBackend"]
