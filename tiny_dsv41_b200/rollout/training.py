"""Exact training records exchanged between samplers and the learner.

The JSON form is the interface of ``rollout_manager/training.py:58-351`` (records written by
either side load in the other):

* ``PolicyRef`` - the activation receipt a sample was drawn under: ``version``, ``digest`` (sha256
  of the policy artifact), run ``lineage``, string ``identities`` and the ``sampling`` profile,
  which must be full categorical sampling (top_p 1, top_k 0) at a positive temperature.
* ``TurnTrace`` - one sampled turn: context ids, action ids, one non-positive behaviour log-prob
  per action, finish reason (eos / stop / length / tool_calls) and stop-token count.
* ``TrainingTrajectory`` - consecutive turns under one policy and a reward (``None`` only for an
  excluded sample, which must give a reason); ``initial_context_sha256`` is the digest of the
  first context.
* ``TrainingGroup`` - exactly ``expected_size`` (>= 2) eligible trajectories of one task,
  context, reset and policy, sample indices 0..G-1, unique request ids.

Here every record class lists its wire fields and which of them hold nested records
(``_NESTED``); one generic encoder / decoder serves all four, and each class keeps its rules in
``_validate``. ``dumps`` / ``loads`` wrap a record as ``{"schema_version": 1, "kind": ...,
"record": ...}`` with sorted keys and compact separators; ``loads`` rejects duplicate keys and
non-finite numbers. Records pickle as their validated dict form.
"""

from __future__ import annotations

import dataclasses
import hashlib
import json
import math
import re
from dataclasses import dataclass, field
from types import MappingProxyType
from typing import Any, Mapping, Sequence

SCHEMA_VERSION = 1
FINISH_REASONS = frozenset({"eos", "stop", "length", "tool_calls"})
_SHA256 = re.compile(r"[0-9a-f]{64}")
_SAMPLING_KEYS = ("temperature", "top_p", "top_k")


# -- value checks ---------------------------------------------------------------------------------
def _fail(message: str):
    raise ValueError(message)


def _whole(value, what: str, minimum: int = 0) -> int:
    if type(value) is int and value >= minimum:
        return value
    _fail(f"{what} must be an integer >= {minimum}")


def _sha(value, what: str) -> str:
    if isinstance(value, str) and _SHA256.fullmatch(value):
        return value
    _fail(f"{what} must be a lowercase SHA256 digest")


def _finite(value, what: str) -> float:
    if type(value) in (int, float) and math.isfinite(value):
        return float(value)
    _fail(f"{what} must be finite")


def _text(value) -> bool:
    return isinstance(value, str) and bool(value)


def _ids(values, what: str) -> tuple[int, ...]:
    if isinstance(values, (str, bytes)):
        _fail(f"{what} requires exact token IDs")
    ids = tuple(values)
    if ids and all(type(v) is int and v >= 0 for v in ids):
        return ids
    _fail(f"{what} requires nonempty nonnegative integer token IDs")


def _fields_exactly(value, names) -> dict:
    if isinstance(value, dict) and set(value) == set(names):
        return value
    _fail("training record has missing or unknown fields")


def token_digest(tokens: Sequence[int]) -> str:
    """sha256 of the compact JSON array of the token ids."""
    return hashlib.sha256(json.dumps(list(_ids(tokens, "tokens")), separators=(",", ":")).encode()).hexdigest()


# -- generic record codec -------------------------------------------------------------------------
class _Record:
    _NESTED: dict[str, tuple[type, bool]] = {}  # field -> (record class, is a sequence)

    def __post_init__(self):
        self._validate()

    def _set(self, name: str, value) -> None:
        object.__setattr__(self, name, value)

    @classmethod
    def _wire_fields(cls) -> list[str]:
        return [f.name for f in dataclasses.fields(cls)]

    def to_dict(self) -> dict:
        out = {}
        for name in self._wire_fields():
            value = getattr(self, name)
            if isinstance(value, _Record):
                value = value.to_dict()
            elif isinstance(value, Mapping):
                value = dict(value)
            elif isinstance(value, tuple):
                value = [v.to_dict() if isinstance(v, _Record) else v for v in value]
            out[name] = value
        return out

    @classmethod
    def from_dict(cls, value):
        values = dict(_fields_exactly(value, cls._wire_fields()))
        for name, (kind, many) in cls._NESTED.items():
            values[name] = [kind.from_dict(v) for v in values[name]] if many else kind.from_dict(values[name])
        return cls(**values)

    def __reduce__(self):
        return type(self).from_dict, (self.to_dict(),)


@dataclass(frozen=True)
class PolicyRef(_Record):
    version: int
    digest: str
    lineage: str
    identities: Mapping[str, str] = field(default_factory=dict)
    sampling: Mapping[str, Any] = field(default_factory=lambda: {"temperature": 1.0, "top_p": 1.0, "top_k": 0})

    def _validate(self):
        _whole(self.version, "policy version")
        _sha(self.digest, "policy digest")
        if not _text(self.lineage):
            _fail("policy requires run lineage")
        identities = dict(self.identities)
        if not all(_text(k) and _text(v) for k, v in identities.items()):
            _fail("policy identities require nonempty string names and values")
        sampling = _fields_exactly(dict(self.sampling), _SAMPLING_KEYS)
        temperature = _finite(sampling["temperature"], "temperature")
        top_p, top_k = sampling["top_p"], sampling["top_k"]
        categorical = type(top_p) in (int, float) and top_p == 1 and type(top_k) is int and top_k == 0
        if temperature <= 0 or not categorical:
            _fail("training requires positive temperature and full categorical sampling")
        self._set("identities", MappingProxyType(identities))
        self._set("sampling", MappingProxyType({"temperature": temperature, "top_p": 1.0, "top_k": 0}))


@dataclass(frozen=True)
class TurnTrace(_Record):
    turn_id: int
    request_id: str
    context_token_ids: Sequence[int]
    action_token_ids: Sequence[int]
    behavior_log_probs: Sequence[float]
    policy: PolicyRef
    finish_reason: str = "stop"
    stop_token_count: int = 0
    context_truncation: str = "none"

    _NESTED = {"policy": (PolicyRef, False)}

    def _validate(self):
        _whole(self.turn_id, "turn_id", 1)
        if not _text(self.request_id):
            _fail("turn requires a request identity")
        if not isinstance(self.policy, PolicyRef):
            _fail("turn requires an actual policy receipt")
        context = _ids(self.context_token_ids, "context_token_ids")
        actions = _ids(self.action_token_ids, "action_token_ids")
        log_probs = tuple(_finite(v, "behavior log probability") for v in self.behavior_log_probs)
        if len(log_probs) != len(actions) or max(log_probs, default=0.0) > 0:
            _fail("each action token requires one nonpositive behavior log probability")
        if self.finish_reason not in FINISH_REASONS:
            _fail("unsupported sampled finish reason")
        if _whole(self.stop_token_count, "stop_token_count") > len(actions):
            _fail("stop_token_count exceeds sampled actions")
        if not _text(self.context_truncation):
            _fail("context truncation rule must be explicit")
        self._set("context_token_ids", context)
        self._set("action_token_ids", actions)
        self._set("behavior_log_probs", log_probs)


@dataclass(frozen=True)
class TrainingTrajectory(_Record):
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

    _NESTED = {"turns": (TurnTrace, True)}

    def _validate(self):
        _whole(self.group_id, "training group_id")
        _whole(self.sample_index, "sample_index")
        if not _text(self.task_id):
            _fail("trajectory requires task identity")
        _sha(self.initial_context_sha256, "initial context digest")
        _sha(self.reset_sha256, "reset digest")
        turns = tuple(self.turns)
        self._check_turns(turns)
        if type(self.reward_eligible) is not bool:
            _fail("reward eligibility must be explicit")
        for name, what in (("reward", "reward"), ("raw_reward", "raw reward")):
            if getattr(self, name) is not None:
                self._set(name, _finite(getattr(self, name), what))
        if self.reward_eligible and self.exclusion_reason is not None:
            _fail("eligible trajectory cannot have an exclusion reason")
        if not self.reward_eligible and not _text(self.exclusion_reason):
            _fail("excluded trajectory requires a reason")
        if self.sampling_seed is not None:
            _whole(self.sampling_seed, "sampling_seed")
        sample_id = f"{self.group_id}:{self.sample_index}" if self.sample_id is None else self.sample_id
        if not _text(sample_id):
            _fail("trajectory requires sample identity")
        # evidence must be plain, finite JSON; keep a frozen deep copy
        self._set("evidence", MappingProxyType(json.loads(json.dumps(dict(self.evidence), allow_nan=False))))
        self._set("sample_id", sample_id)
        self._set("turns", turns)

    def _check_turns(self, turns) -> None:
        if not turns or not all(isinstance(t, TurnTrace) for t in turns):
            _fail("trajectory requires exact turn traces")
        if [t.turn_id for t in turns] != list(range(1, len(turns) + 1)):
            _fail("trajectory turn IDs must be consecutive and ordered")
        if len({t.request_id for t in turns}) < len(turns):
            _fail("trajectory has duplicate request identities")
        if any(t.policy != turns[0].policy for t in turns[1:]):
            _fail("all trajectory turns require one policy receipt")
        if token_digest(turns[0].context_token_ids) != self.initial_context_sha256:
            _fail("initial context digest differs from actual tokens")

    # -- views ------------------------------------------------------------------------------------
    @property
    def policy(self) -> PolicyRef:
        return self.turns[0].policy

    @property
    def policy_version(self) -> int:
        return self.policy.version

    @property
    def behavior_log_probs(self) -> list[float]:
        return [v for turn in self.turns for v in turn.behavior_log_probs]

    @property
    def finish_reason(self) -> str:
        return self.turns[-1].finish_reason

    @property
    def stop_token_count(self) -> int:
        return self.turns[-1].stop_token_count

    def single_turn(self) -> TurnTrace:
        if len(self.turns) == 1:
            return self.turns[0]
        _fail("multi-turn trajectories require per-turn contexts, not flattened responses")

    @property
    def prompt_ids(self) -> list[int]:
        return list(self.single_turn().context_token_ids)

    @property
    def response_ids(self) -> list[int]:
        return list(self.single_turn().action_token_ids)

    @property
    def content_ids(self) -> list[int]:
        """The response without its trailing stop tokens."""
        response = self.response_ids
        return response[:len(response) - self.stop_token_count]


@dataclass(frozen=True)
class TrainingGroup(_Record):
    group_id: int
    task_id: str
    initial_context_sha256: str
    reset_sha256: str
    policy: PolicyRef
    expected_size: int
    samples: Sequence[TrainingTrajectory]

    _NESTED = {"policy": (PolicyRef, False), "samples": (TrainingTrajectory, True)}

    def _validate(self):
        _whole(self.group_id, "training group_id")
        size = _whole(self.expected_size, "expected group size", 2)
        samples = tuple(self.samples)
        if len(samples) != size or not all(isinstance(s, TrainingTrajectory) for s in samples):
            _fail("training requires a complete group of exactly G trajectories")
        indices_ok = sorted(s.sample_index for s in samples) == list(range(size))
        if not indices_ok or len({s.sample_id for s in samples}) != size:
            _fail("training group requires unique sample identities and indices 0..G-1")
        requests = [turn.request_id for s in samples for turn in s.turns]
        if len(set(requests)) != len(requests):
            _fail("training group has duplicate request identities")
        shared = (self.group_id, self.task_id, self.initial_context_sha256, self.reset_sha256, self.policy)
        for s in samples:
            if (s.group_id, s.task_id, s.initial_context_sha256, s.reset_sha256, s.policy) != shared:
                _fail("training group requires the same task, initial context, reset and policy")
            if s.reward is None or not s.reward_eligible:
                _fail("training requires G eligible finite rewards; missing is not zero")
        self._set("samples", tuple(sorted(samples, key=lambda s: s.sample_index)))

    @property
    def policy_version(self) -> int:
        return self.policy.version


# -- framed JSON ----------------------------------------------------------------------------------
_KINDS = {cls.__name__: cls for cls in (PolicyRef, TurnTrace, TrainingTrajectory, TrainingGroup)}


def dumps(record) -> str:
    kind = type(record).__name__
    if _KINDS.get(kind) is not type(record):
        raise TypeError("unsupported training record")
    frame = {"schema_version": SCHEMA_VERSION, "kind": kind, "record": record.to_dict()}
    return json.dumps(frame, sort_keys=True, separators=(",", ":"), allow_nan=False)


def _unique_keys(pairs):
    keys = [key for key, _ in pairs]
    if len(set(keys)) != len(keys):
        raise ValueError("duplicate JSON field")
    return dict(pairs)


def _no_constants(name):
    raise ValueError("nonfinite JSON number")


def loads(text: str):
    frame = _fields_exactly(json.loads(text, object_pairs_hook=_unique_keys, parse_constant=_no_constants),
                            ("schema_version", "kind", "record"))
    version = frame["schema_version"]
    if type(version) is not int or version != SCHEMA_VERSION or frame["kind"] not in _KINDS:
        raise ValueError("unsupported training record schema or kind")
    return _KINDS[frame["kind"]].from_dict(frame["record"])


# -- native rollout groups ------------------------------------------------------------------------
def from_rollout_group(group, policy: PolicyRef, task_id: str, reset_sha256: str, *, request_prefix=None):
    """A native ``RolloutGroup`` as a single-turn ``TrainingGroup`` (no probability is recomputed)."""
    if group.policy_version != policy.version:
        raise ValueError("legacy group differs from acknowledged policy version")
    if len(group.samples) < 2:
        raise ValueError("training requires a complete group of at least two samples")
    if request_prefix is None:
        request_prefix = f"{hashlib.sha256(policy.lineage.encode()).hexdigest()[:12]}-g{group.group_id}"
    context = token_digest(group.samples[0].prompt_ids)
    trajectories = []
    for index, sample in enumerate(group.samples):
        if sample.policy_version != policy.version:
            raise ValueError("legacy sample differs from acknowledged policy version")
        turn = TurnTrace(1, f"{request_prefix}-s{index}", sample.prompt_ids, sample.response_ids,
                         sample.behavior_log_probs, policy, sample.finish_reason, sample.stop_token_count)
        trajectories.append(TrainingTrajectory(group.group_id, task_id, context, reset_sha256, index, (turn,),
                                               sample.reward, raw_reward=sample.raw_reward))
    return TrainingGroup(group.group_id, task_id, context, reset_sha256, policy, len(trajectories), trajectories)


def to_rollout_group(group: TrainingGroup):
    """A single-turn ``TrainingGroup`` as the native ``RolloutGroup``."""
    from ..rl.rollout import RolloutGroup, Sample

    samples = []
    for trajectory in group.samples:
        turn = trajectory.single_turn()
        if turn.finish_reason == "tool_calls":
            raise ValueError("legacy Sample does not represent tool-call finish reasons")
        samples.append(Sample(list(turn.context_token_ids), list(turn.action_token_ids),
                              list(turn.behavior_log_probs), trajectory.reward, trajectory.policy_version,
                              turn.finish_reason, turn.stop_token_count, trajectory.raw_reward))
    return RolloutGroup(samples, group.group_id, group.policy_version)


__all__ = ["FINISH_REASONS", "PolicyRef", "SCHEMA_VERSION", "TrainingGroup", "TrainingTrajectory", "TurnTrace",
           "dumps", "from_rollout_group", "loads", "to_rollout_group", "token_digest"]
