"""Benchmark episodes into GRPO training groups (the accounting half of
``rollout_manager/benchmark_training.py`` of the reference).

A semantic group is G >= 2 episodes of one task, one benchmark pass and one leased policy. The
caller registers the prepared plans, then hands each finished ``EpisodeResult`` to
``GroupAssembler.complete``; when the last episode of a group arrives it returns either a
``TrainingGroup`` (every sample eligible, scored by the declared reward mapping, its sampled turns
carrying the lease's policy receipt and durable, validated request records) or a
``GroupExclusion`` with one reason per failing sample. Admission and execution stay with the
rollout coordinator; the capacities here only bound the bookkeeping.
"""

from __future__ import annotations

import hashlib
import json
import math
from collections.abc import Mapping, Sequence
from dataclasses import asdict, dataclass

from .contracts import EpisodePlan, EpisodeResult, request_uncertain
from .training import PolicyRef, TrainingGroup, TrainingTrajectory, TurnTrace

# benchmark -> the one reward mapping version it supports
REWARD_MAPPINGS = {"kernelbench": "native-final-correctness-v1", "cuda-agent": "native-final-correctness-v1",
                   "terminal-bench": "terminal-validated-verifier-v1"}


def _is_sha256(value) -> bool:
    return isinstance(value, str) and len(value) == 64 and all(c in "0123456789abcdef" for c in value)


@dataclass(frozen=True)
class RewardPolicy:
    benchmark: str
    mapping: str

    def __post_init__(self):
        if REWARD_MAPPINGS.get(self.benchmark) != self.mapping:
            raise ValueError("declare the supported, versioned reward mapping of the benchmark")

    def reward(self, result: EpisodeResult) -> float:
        """The scalar reward of a completed, verified and cleaned-up episode; raises otherwise."""
        if result.identity.benchmark != self.benchmark:
            raise ValueError("episode of another benchmark")
        if (result.execution_state != "completed" or not result.score_eligible
                or result.failure_category is not None):
            raise ValueError("episode did not complete as a score-eligible run")
        if result.cleanup_state not in ("verified", "not_required"):
            raise ValueError("episode cleanup is unproven")
        if not result.request_state or request_uncertain(result.request_state):
            raise ValueError("episode lacks durable request completion records")
        outcome = result.native_outcome
        if outcome.get("training_evidence_error"):
            raise ValueError("the backend rejected the training evidence")
        if self.mapping == "native-final-correctness-v1":
            correct = outcome.get("final_correct")
            if type(correct) is not bool or result.verification_state != ("passed" if correct else "failed"):
                raise ValueError("final verification is missing or disagrees with the outcome")
            return 1.0 if correct else 0.0
        if result.verification_state != "evaluated" or outcome.get("review_classification") != "evaluated":
            raise ValueError("the verifier has no authoritative evaluated result")
        value = outcome.get("validated_reported_reward")
        if type(value) not in (int, float) or not math.isfinite(value):
            raise ValueError("the verifier reward is missing or not finite")
        return float(value)


@dataclass(frozen=True)
class GroupRegistration:
    group_id: int
    plans: Sequence[EpisodePlan]
    policy: PolicyRef
    initial_context_sha256: str
    reset_sha256: str
    reward_policy: RewardPolicy

    def __post_init__(self):
        plans = tuple(self.plans)
        if type(self.group_id) is not int or self.group_id < 0 or len(plans) < 2:
            raise ValueError("a training group needs a nonnegative integer id and G >= 2 plans")
        if not all(isinstance(p, EpisodePlan) for p in plans) or not isinstance(self.policy, PolicyRef):
            raise ValueError("a group registration takes prepared plans and a policy lease")
        if len({p.identity for p in plans}) != len(plans):
            raise ValueError("episode identities within a group must be distinct")
        if sorted(p.identity.sample_index for p in plans) != list(range(len(plans))):
            raise ValueError("sample indices of a group must be exactly 0..G-1")
        tasks = {(p.identity.run_id, p.identity.benchmark, p.identity.pass_index, p.task.task_id, p.task.source_sha256)
                 for p in plans}
        if len(tasks) != 1:
            raise ValueError("a semantic group holds one task of one pass of one run")
        if self.reward_policy.benchmark != plans[0].identity.benchmark:
            raise ValueError("the reward mapping is for another benchmark")
        if not (_is_sha256(self.initial_context_sha256) and _is_sha256(self.reset_sha256)):
            raise ValueError("initial context and reset need exact sha256 identities")
        object.__setattr__(self, "plans", tuple(sorted(plans, key=lambda p: p.identity.sample_index)))


@dataclass(frozen=True)
class GroupExclusion:
    group_id: int
    expected_size: int
    reasons: tuple[str, ...]
    episodes: tuple[EpisodeResult, ...]

    def to_dict(self) -> dict:
        return {"schema_version": 1, "kind": "excluded_training_group", "group_id": self.group_id,
                "expected_size": self.expected_size, "reasons": list(self.reasons),
                "episodes": [asdict(e) for e in self.episodes]}


def _sample(registration: GroupRegistration, plan: EpisodePlan, episode: EpisodeResult) -> TrainingTrajectory:
    if episode.source_sha256 != plan.task.source_sha256:
        raise ValueError("the completed source digest differs from the registered task")
    reward = registration.reward_policy.reward(episode)
    raw_turns = episode.native_outcome.get("training_turns")
    if not isinstance(raw_turns, (list, tuple)) or not raw_turns:
        raise ValueError("the exact sampled training turns are missing")
    turns = tuple(TurnTrace.from_dict(t) for t in raw_turns)
    if any(t.policy != registration.policy for t in turns):
        raise ValueError("a turn's policy receipt differs from the group lease")
    records = episode.request_state.get("requests")
    if not isinstance(records, Mapping):
        raise ValueError("the sampled requests have no delivery records")
    for t in turns:
        record = records.get(t.request_id)
        if (not isinstance(record, Mapping) or record.get("state") != "response_received"
                or record.get("training_evidence") != "validated"):
            raise ValueError("a sampled request lacks a durable response with validated training evidence")
    identity = plan.identity
    return TrainingTrajectory(
        registration.group_id, plan.task.task_id, registration.initial_context_sha256, registration.reset_sha256,
        identity.sample_index, turns, reward,
        evidence={"episode_identity": asdict(episode.identity), "native_artifacts": episode.native_artifacts,
                  "native_outcome": dict(episode.native_outcome), "reward_mapping": registration.reward_policy.mapping},
        sample_id=identity.trial_id or f"{identity.run_id}:{registration.group_id}:{identity.sample_index}",
        raw_reward=reward, sampling_seed=identity.sampling_seed)


class GroupAssembler:
    """Bounded bookkeeping from registered plans to finished groups."""

    def __init__(self, *, max_groups: int = 1, max_episodes: int = 8) -> None:
        if type(max_groups) is not int or max_groups < 1 or type(max_episodes) is not int or max_episodes < 2:
            raise ValueError("assembler capacities: max_groups >= 1, max_episodes >= 2")
        self.max_groups, self.max_episodes = max_groups, max_episodes
        self._groups: dict[int, dict] = {}
        self._owner: dict = {}
        self._last_group = -1

    def register(self, registration: GroupRegistration) -> None:
        if not isinstance(registration, GroupRegistration) or registration.group_id <= self._last_group:
            raise ValueError("register a new group id, larger than every earlier one")
        if (len(self._groups) >= self.max_groups
                or len(self._owner) + len(registration.plans) > self.max_episodes):
            raise ValueError("the assembler's group capacity is exhausted")
        if any(p.identity in self._owner for p in registration.plans):
            raise ValueError("an episode may belong to one training group only")
        self._groups[registration.group_id] = {"registration": registration, "results": {}}
        for p in registration.plans:
            self._owner[p.identity] = registration.group_id
        self._last_group = registration.group_id

    def complete(self, result: EpisodeResult):
        """Record one finished episode; returns the group's TrainingGroup / GroupExclusion when it
        was the last one, else None."""
        if not isinstance(result, EpisodeResult) or result.identity not in self._owner:
            raise ValueError("the result was never registered or is already accounted for")
        group_id = self._owner[result.identity]
        row = self._groups[group_id]
        if result.identity in row["results"]:
            raise ValueError("duplicate completion of an episode")
        row["results"][result.identity] = result
        registration = row["registration"]
        if len(row["results"]) < len(registration.plans):
            return None
        episodes = tuple(row["results"][p.identity] for p in registration.plans)
        samples, reasons = [], []
        for plan, episode in zip(registration.plans, episodes):
            try:
                samples.append(_sample(registration, plan, episode))
            except (KeyError, TypeError, ValueError) as error:
                reasons.append(f"sample-{plan.identity.sample_index}: {error}")
        try:
            receipt = (TrainingGroup(group_id, registration.plans[0].task.task_id, registration.initial_context_sha256,
                                     registration.reset_sha256, registration.policy, len(registration.plans), samples)
                       if not reasons else GroupExclusion(group_id, len(registration.plans), tuple(reasons), episodes))
        except ValueError as error:
            receipt = GroupExclusion(group_id, len(registration.plans), (str(error),), episodes)
        for p in registration.plans:
            del self._owner[p.identity]
        del self._groups[group_id]
        return receipt


def artifact_policy(artifact: Mapping, *, identities: Mapping[str, str] | None = None) -> PolicyRef:
    """The PolicyRef of a published policy artifact (its run identity hashed in); external routes
    add their qualified tokenizer / chat-template hashes through ``identities``."""
    identity = json.dumps(artifact["identity"], sort_keys=True, separators=(",", ":"), allow_nan=False).encode()
    return PolicyRef(artifact["version"], artifact["digest"], artifact["lineage"],
                     {**(identities or {}), "run_identity_sha256": hashlib.sha256(identity).hexdigest()},
                     artifact["sampling"])


__all__ = ["GroupAssembler", "GroupExclusion", "GroupRegistration", "REWARD_MAPPINGS", "RewardPolicy",
           "artifact_policy"]
