"""Exact training records exchanged between samplers and the learner.

The JSON format is the reference's (``rollout_manager/training.py:58-351``), so records written
by either side load in the other:

* ``PolicyRef``: the activation receipt a sample was drawn under - ``version``, ``digest``
  (sha256 of the policy artifact), run ``lineage``, string ``identities`` and the ``sampling``
  profile, which must be full categorical sampling (top_p 1, top_k 0) at a positive temperature.
* ``TurnTrace``: one sampled turn - context ids, action ids, one non-positive behaviour
  log-prob per action, finish reason (eos / stop / length / tool_calls), stop-token count.
* ``TrainingTrajectory``: consecutive turns under one policy, a reward (``None`` only when the
  sample is excluded, with a reason), ``initial_context_sha256 == token_digest(first context)``.
* ``TrainingGroup``: exactly ``expected_size`` (>= 2) eligible trajectories of one task / context
  / reset / policy, sample indices 0..G-1, unique request ids.

``dumps``/``loads`` wrap a record as ``{"schema_version": 1, "kind": ..., "record": ...}`` with
sorted keys and compact separators; ``loads`` rejects duplicate keys and non-finite numbers.
"""

from __future__ import annotations

import hashlib
import json
import math
import re
from dataclasses import dataclass, field
from types import MappingProxyType
from typing import Any, Mapping, Sequence

SCHEMA_VERSION = 1
_SHA256 = re.compile(r"[0-9a-f]{64}")
_DEFAULT_SAMPLING = {"temperature": 1.0, "top_p": 1.0, "top_k": 0}


def _check_int(value, what: str, minimum: int = 0) -> None:
    if type(value) is not int or value < minimum:
        raise ValueError(f"{what} must be an integer >= {minimum}")


def _check_sha(value, what: str) -> None:
    if not isinstance(value, str) or not _SHA256.fullmatch(value):
        raise ValueError(f"{what} must be a lowercase SHA256 digest")


def _token_tuple(values, what: str) -> tuple[int, ...]:
    if isinstance(values, (str, bytes)):
        raise ValueError(f"{what} requires exact token IDs")
    out = tuple(values)
    if not out or any(type(v) is not int or v < 0 for v in out):
        raise ValueError(f"{what} requires nonempty nonnegative integer token IDs")
    return out


def _finite_float(value, what: str) -> float:
    if type(value) not in (int, float) or not math.isfinite(value):
        raise ValueError(f"{what} must be finite")
    return float(value)


def _exact_fields(value, names) -> None:
    if not isinstance(value, dict) or set(value) != set(names):
        raise ValueError("training record has missing or unknown fields")


def token_digest(tokens: Sequence[int]) -> str:
    ids = list(_token_tuple(tokens, "tokens"))
    return hashlib.sha256(json.dumps(ids, separators=(",", ":")).encode()).hexdigest()


class _Pickles:
    """Records travel between processes as their validated dict form."""

    def __reduce__(self):
        return type(self).from_dict, (self.to_dict(),)


@dataclass(frozen=True)
class PolicyRef(_Pickles):
    version: int
    digest: str
    lineage: str
    identities: Mapping[str, str] = field(default_factory=dict)
    sampling: Mapping[str, Any] = field(default_factory=lambda: dict(_DEFAULT_SAMPLING))

    def __post_init__(self):
        _check_int(self.version, "policy version")
        _check_sha(self.digest, "policy digest")
        if not isinstance(self.lineage, str) or not self.lineage:
            raise ValueError("policy requires run lineage")
        ids = dict(self.identities)
        if any(not (isinstance(k, str) and k and isinstance(v, str) and v) for k, v in ids.items()):
            raise ValueError("policy identities require nonempty string names and values")
        sampling = dict(self.sampling)
        _exact_fields(sampling, ("temperature", "top_p", "top_k"))
        temperature = _finite_float(sampling["temperature"], "temperature")
        full = (type(sampling["top_p"]) in (int, float) and sampling["top_p"] == 1
                and type(sampling["top_k"]) is int and sampling["top_k"] == 0)
        if temperature <= 0 or not full:
            raise ValueError("training requires positive temperature and full categorical sampling")
        object.__setattr__(self, "identities", MappingProxyType(ids))
        object.__setattr__(self, "sampling", MappingProxyType({"temperature": temperature, "top_p": 1.0, "top_k": 0}))

    def to_dict(self) -> dict:
        return {"version": self.version, "digest": self.digest, "lineage": self.lineage,
                "identities": dict(self.identities), "sampling": dict(self.sampling)}

    @classmethod
    def from_dict(cls, value) -> "PolicyRef":
        _exact_fields(value, ("version", "digest", "lineage", "identities", "sampling"))
        return cls(**value)


@dataclass(frozen=True)
class TurnTrace(_Pickles):
    turn_id: int
    request_id: str
    context_token_ids: Sequence[int]
    action_token_ids: Sequence[int]
    behavior_log_probs: Sequence[float]
    policy: PolicyRef
    finish_reason: str = "stop"
    stop_token_count: int = 0
    context_truncation: str = "none"

    def __post_init__(self):
        _check_int(self.turn_id, "turn_id", 1)
        if not isinstance(self.request_id, str) or not self.request_id:
            raise ValueError("turn requires a request identity")
        if not isinstance(self.policy, PolicyRef):
            raise ValueError("turn requires an actual policy receipt")
        context = _token_tuple(self.context_token_ids, "context_token_ids")
        actions = _token_tuple(self.action_token_ids, "action_token_ids")
        logps = tuple(_finite_float(v, "behavior log probability") for v in self.behavior_log_probs)
        if len(actions) != len(logps) or any(v > 0 for v in logps):
            raise ValueError("each action token requires one nonpositive behavior log probability")
        if self.finish_reason not in {"eos", "stop", "length", "tool_calls"}:
            raise ValueError("unsupported sampled finish reason")
        _check_int(self.stop_token_count, "stop_token_count")
        if self.stop_token_count > len(actions):
            raise ValueError("stop_token_count exceeds sampled actions")
        if not isinstance(self.context_truncation, str) or not self.context_truncation:
            raise ValueError("context truncation rule must be explicit")
        object.__setattr__(self, "context_token_ids", context)
        object.__setattr__(self, "action_token_ids", actions)
        object.__setattr__(self, "behavior_log_probs", logps)

    def to_dict(self) -> dict:
        return {"turn_id": self.turn_id, "request_id": self.request_id,
                "context_token_ids": list(self.context_token_ids), "action_token_ids": list(self.action_token_ids),
                "behavior_log_probs": list(self.behavior_log_probs), "policy": self.policy.to_dict(),
                "finish_reason": self.finish_reason, "stop_token_count": self.stop_token_count,
                "context_truncation": self.context_truncation}

    @classmethod
    def from_dict(cls, value) -> "TurnTrace":
        _exact_fields(value, cls.__dataclass_fields__)
        return cls(**{**value, "policy": PolicyRef.from_dict(value["policy"])})


@dataclass(frozen=True)
class TrainingTrajectory(_Pickles):
    group_id: int
    task_id: str
    initial_context_sha256: str
    reset_sha256: str
    sample_index: int
    turns: Sequence[TurnTrace]
    reward: float | None
    reward_eligible: bool = True
    exclusion_reason: str | None = None
    evidence: Mapping[str, Any] = field(default_factory=dict)
    sample_id: str | None = None
    raw_reward: float | None = None
    sampling_seed: int | None = None

    def __post_init__(self):
        _check_int(self.group_id, "training group_id")
        _check_int(self.sample_index, "sample_index")
        if not isinstance(self.task_id, str) or not self.task_id:
            raise ValueError("trajectory requires task identity")
        _check_sha(self.initial_context_sha256, "initial context digest")
        _check_sha(self.reset_sha256, "reset digest")
        turns = tuple(self.turns)
        if not turns or any(not isinstance(t, TurnTrace) for t in turns):
            raise ValueError("trajectory requires exact turn traces")
        if [t.turn_id for t in turns] != list(range(1, len(turns) + 1)):
            raise ValueError("trajectory turn IDs must be consecutive and ordered")
        if len({t.request_id for t in turns}) != len(turns):
            raise ValueError("trajectory has duplicate request identities")
        if any(t.policy != turns[0].policy for t in turns):
            raise ValueError("all trajectory turns require one policy receipt")
        if token_digest(turns[0].context_token_ids) != self.initial_context_sha256:
            raise ValueError("initial context digest differs from actual tokens")
        if type(self.reward_eligible) is not bool:
            raise ValueError("reward eligibility must be explicit")
        if self.reward is not None:
            object.__setattr__(self, "reward", _finite_float(self.reward, "reward"))
        if self.raw_reward is not None:
            object.__setattr__(self, "raw_reward", _finite_float(self.raw_reward, "raw reward"))
        if not self.reward_eligible and not (isinstance(self.exclusion_reason, str) and self.exclusion_reason):
            raise ValueError("excluded trajectory requires a reason")
        if self.reward_eligible and self.exclusion_reason is not None:
            raise ValueError("eligible trajectory cannot have an exclusion reason")
        if self.sampling_seed is not None:
            _check_int(self.sampling_seed, "sampling_seed")
        sample_id = self.sample_id if self.sample_id is not None else f"{self.group_id}:{self.sample_index}"
        if not isinstance(sample_id, str) or not sample_id:
            raise ValueError("trajectory requires sample identity")
        evidence = json.loads(json.dumps(dict(self.evidence), allow_nan=False))
        object.__setattr__(self, "evidence", MappingProxyType(evidence))
        object.__setattr__(self, "sample_id", sample_id)
        object.__setattr__(self, "turns", turns)

    @property
    def policy(self) -> PolicyRef:
        return self.turns[0].policy

    @property
    def policy_version(self) -> int:
        return self.policy.version

    @property
    def behavior_log_probs(self) -> list[float]:
        return [v for t in self.turns for v in t.behavior_log_probs]

    @property
    def finish_reason(self) -> str:
        return self.turns[-1].finish_reason

    @property
    def stop_token_count(self) -> int:
        return self.turns[-1].stop_token_count

    def single_turn(self) -> TurnTrace:
        if len(self.turns) != 1:
            raise ValueError("multi-turn trajectories require per-turn contexts, not flattened responses")
        return self.turns[0]

    @property
    def prompt_ids(self) -> list[int]:
        return list(self.single_turn().context_token_ids)

    @property
    def response_ids(self) -> list[int]:
        return list(self.single_turn().action_token_ids)

    @property
    def content_ids(self) -> list[int]:
        r = self.response_ids
        return r[:-self.stop_token_count] if self.stop_token_count else r

    def to_dict(self) -> dict:
        return {"group_id": self.group_id, "task_id": self.task_id,
                "initial_context_sha256": self.initial_context_sha256, "reset_sha256": self.reset_sha256,
                "sample_index": self.sample_index, "sample_id": self.sample_id,
                "turns": [t.to_dict() for t in self.turns], "reward": self.reward,
                "reward_eligible": self.reward_eligible, "exclusion_reason": self.exclusion_reason,
                "evidence": dict(self.evidence), "raw_reward": self.raw_reward, "sampling_seed": self.sampling_seed}

    @classmethod
    def from_dict(cls, value) -> "TrainingTrajectory":
        _exact_fields(value, cls.__dataclass_fields__)
        return cls(**{**value, "turns": [TurnTrace.from_dict(t) for t in value["turns"]]})


@dataclass(frozen=True)
class TrainingGroup(_Pickles):
    group_id: int
    task_id: str
    initial_context_sha256: str
    reset_sha256: str
    policy: PolicyRef
    expected_size: int
    samples: Sequence[TrainingTrajectory]

    def __post_init__(self):
        _check_int(self.group_id, "training group_id")
        _check_int(self.expected_size, "expected group size", 2)
        samples = tuple(self.samples)
        if len(samples) != self.expected_size or any(not isinstance(s, TrainingTrajectory) for s in samples):
            raise ValueError("training requires a complete group of exactly G trajectories")
        if ({s.sample_index for s in samples} != set(range(self.expected_size))
                or len({s.sample_id for s in samples}) != self.expected_size):
            raise ValueError("training group requires unique sample identities and indices 0..G-1")
        requests = [t.request_id for s in samples for t in s.turns]
        if len(set(requests)) != len(requests):
            raise ValueError("training group has duplicate request identities")
        key = (self.group_id, self.task_id, self.initial_context_sha256, self.reset_sha256, self.policy)
        for s in samples:
            if (s.group_id, s.task_id, s.initial_context_sha256, s.reset_sha256, s.policy) != key:
                raise ValueError("training group requires the same task, initial context, reset and policy")
            if not s.reward_eligible or s.reward is None:
                raise ValueError("training requires G eligible finite rewards; missing is not zero")
        object.__setattr__(self, "samples", tuple(sorted(samples, key=lambda s: s.sample_index)))

    @property
    def policy_version(self) -> int:
        return self.policy.version

    def to_dict(self) -> dict:
        return {"group_id": self.group_id, "task_id": self.task_id,
                "initial_context_sha256": self.initial_context_sha256, "reset_sha256": self.reset_sha256,
                "policy": self.policy.to_dict(), "expected_size": self.expected_size,
                "samples": [s.to_dict() for s in self.samples]}

    @classmethod
    def from_dict(cls, value) -> "TrainingGroup":
        _exact_fields(value, cls.__dataclass_fields__)
        return cls(**{**value, "policy": PolicyRef.from_dict(value["policy"]),
                      "samples": [TrainingTrajectory.from_dict(s) for s in value["samples"]]})


_KINDS = {c.__name__: c for c in (PolicyRef, TurnTrace, TrainingTrajectory, TrainingGroup)}


def dumps(record) -> str:
    kind = type(record).__name__
    if _KINDS.get(kind) is not type(record):
        raise TypeError("unsupported training record")
    return json.dumps({"schema_version": SCHEMA_VERSION, "kind": kind, "record": record.to_dict()},
                      sort_keys=True, separators=(",", ":"), allow_nan=False)


def loads(text: str):
    def no_duplicates(pairs):
        out = {}
        for k, v in pairs:
            if k in out:
                raise ValueError("duplicate JSON field")
            out[k] = v
        return out

    def reject_constant(_):
        raise ValueError("nonfinite JSON number")

    payload = json.loads(text, object_pairs_hook=no_duplicates, parse_constant=reject_constant)
    _exact_fields(payload, ("schema_version", "kind", "record"))
    if type(payload["schema_version"]) is not int or payload["schema_version"] != SCHEMA_VERSION \
            or payload["kind"] not in _KINDS:
        raise ValueError("unsupported training record schema or kind")
    return _KINDS[payload["kind"]].from_dict(payload["record"])


def from_rollout_group(group, policy: PolicyRef, task_id: str, reset_sha256: str, *, request_prefix=None):
    """A native ``RolloutGroup`` as a single-turn ``TrainingGroup`` (no probability is recomputed)."""
    if group.policy_version != policy.version:
        raise ValueError("legacy group differs from acknowledged policy version")
    if len(group.samples) < 2:
        raise ValueError("training requires a complete group of at least two samples")
    context = token_digest(group.samples[0].prompt_ids)
    prefix = request_prefix or hashlib.sha256(policy.lineage.encode()).hexdigest()[:12] + f"-g{group.group_id}"
    samples = []
    for i, s in enumerate(group.samples):
        if s.policy_version != policy.version:
            raise ValueError("legacy sample differs from acknowledged policy version")
        turn = TurnTrace(1, f"{prefix}-s{i}", s.prompt_ids, s.response_ids, s.behavior_log_probs, policy,
                         s.finish_reason, s.stop_token_count)
        samples.append(TrainingTrajectory(group.group_id, task_id, context, reset_sha256, i, (turn,), s.reward,
                                          raw_reward=s.raw_reward))
    return TrainingGroup(group.group_id, task_id, context, reset_sha256, policy, len(samples), samples)


def to_rollout_group(group: TrainingGroup):
    """A single-turn ``TrainingGroup`` as the native ``RolloutGroup``."""
    from ..rl.rollout import RolloutGroup, Sample

    samples = []
    for traj in group.samples:
        turn = traj.single_turn()
        if turn.finish_reason == "tool_calls":
            raise ValueError("legacy Sample does not represent tool-call finish reasons")
        samples.append(Sample(list(turn.context_token_ids), list(turn.action_token_ids), list(turn.behavior_log_probs),
                              traj.reward, traj.policy_version, turn.finish_reason, turn.stop_token_count,
                              traj.raw_reward))
    return RolloutGroup(samples, group.group_id, group.policy_version)


__all__ = ["PolicyRef", "SCHEMA_VERSION", "TrainingGroup", "TrainingTrajectory", "TurnTrace", "dumps",
           "from_rollout_group", "loads", "to_rollout_group", "token_digest"]
