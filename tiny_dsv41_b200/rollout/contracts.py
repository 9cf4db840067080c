"""Contracts between the rollout coordinator, dataset adapters and episode backends.

The dataclass fields are the interface of ``rollout_manager/contracts.py:12-150`` (records cross
the process boundary to the rollout service). A ``TaskSpec`` names one benchmark task with its
pinned source hash, payload and resource needs; an ``EpisodePlan`` is one sample of a task under
an ``EpisodeIdentity``; a backend turns a plan into an ``EpisodeResult``.

``request_uncertain`` answers whether a model request may still be running (or be billed)
remotely. Cancelling locally never proves that a remote request stopped, so an uncertain request
keeps its slot quarantined.
"""

from __future__ import annotations

import math
import threading
from collections import deque
from dataclasses import dataclass, field
from typing import Any, Mapping, Protocol

SCHEMA_VERSION = 1
BENCHMARKS = frozenset({"kernelbench", "cuda-agent", "terminal-bench", "prompt-response"})
# the payload key each benchmark's tasks must carry
_PAYLOAD_KEY = {"terminal-bench": "task_path", "prompt-response": "prompt_response"}
_DEFAULT_PAYLOAD_KEY = "native_case"
ACCOUNTING_SCOPES = ("episode", "backend-stage")


def _require(condition: bool, message: str) -> None:
    if not condition:
        raise ValueError(message)


def _quantity(value: Any) -> bool:
    """A finite, nonnegative number (bools are not quantities)."""
    return not isinstance(value, bool) and isinstance(value, (int, float)) and math.isfinite(value) and value >= 0


@dataclass(frozen=True)
class ResourceRequirements:
    executor: str
    cpu: float = 0
    memory_bytes: int = 0
    storage_bytes: int = 0
    gpu_count: int = 0
    accounting: str = "episode"

    def __post_init__(self):
        _require(bool(self.executor) and self.accounting in ACCOUNTING_SCOPES,
                 "resources require an executor and supported accounting scope")
        _require(all(map(_quantity, (self.cpu, self.memory_bytes, self.storage_bytes, self.gpu_count))),
                 "resource quantities must be finite and nonnegative")


@dataclass(frozen=True)
class TaskSpec:
    benchmark: str
    task_id: str
    source_sha256: str
    payload: Mapping[str, Any]
    resources: ResourceRequirements
    budgets: Mapping[str, Any] = field(default_factory=dict)
    provenance: Mapping[str, Any] = field(default_factory=dict)

    @property
    def payload_key(self) -> str:
        return _PAYLOAD_KEY.get(self.benchmark, _DEFAULT_PAYLOAD_KEY)

    def __post_init__(self):
        _require(self.benchmark in BENCHMARKS and bool(self.task_id) and bool(self.source_sha256),
                 "task requires a supported benchmark, pinned identity and source hash")
        _require(self.payload_key in self.payload, f"{self.benchmark} payload requires {self.payload_key}")
        _require(not (self.benchmark == "terminal-bench" and "code" in self.payload),
                 "Terminal-Bench does not have a CUDA reference-code contract")


@dataclass(frozen=True)
class EpisodeIdentity:
    run_id: str
    benchmark: str
    task_id: str
    group_id: str
    sample_index: int
    pass_index: int = 0
    trial_id: str | None = None
    sampling_seed: int | None = None

    def __post_init__(self):
        _require(bool(self.run_id and self.task_id and self.group_id) and self.benchmark in BENCHMARKS,
                 "episode requires run, benchmark, task and group identities")
        _require(min(self.sample_index, self.pass_index) >= 0, "sample and pass indices must be nonnegative")


@dataclass(frozen=True)
class EpisodePlan:
    identity: EpisodeIdentity
    task: TaskSpec
    payload: Mapping[str, Any] | None = None

    def __post_init__(self):
        same = self.identity.benchmark == self.task.benchmark and self.identity.task_id == self.task.task_id
        _require(same, "episode and task identities disagree")


@dataclass(frozen=True)
class EpisodeResult:
    identity: EpisodeIdentity
    execution_state: str
    verification_state: str
    score_eligible: bool
    cleanup_state: str
    native_outcome: Mapping[str, Any]
    native_artifacts: Any
    usage: Mapping[str, Any] | None = None
    timings: Mapping[str, Any] | None = None
    failure_category: str | None = None
    model_identity: str | None = None
    request_state: Mapping[str, Any] | None = None
    configuration_sha256: str | None = None
    source_sha256: str | None = None


class CancellationToken:
    """Cooperative cancellation shared by asyncio tasks and threads; the first reason is kept."""

    def __init__(self, event: threading.Event | None = None) -> None:
        self.event = threading.Event() if event is None else event
        self.reason: str | None = None
        self._guard = threading.Lock()

    def cancelled(self) -> bool:
        return self.event.is_set()

    def cancel(self, reason: str = "cancelled") -> None:
        with self._guard:
            self.reason = self.reason if self.reason is not None else reason
            self.event.set()


class DatasetAdapter(Protocol):
    def enumerate(self) -> list[TaskSpec]: ...


class EpisodeBackend(Protocol):
    async def execute(self, plan: EpisodePlan, cancellation: CancellationToken) -> EpisodeResult: ...


def _node_uncertain(node: Mapping[str, Any]) -> bool:
    """The rules for one level of a request-state record."""
    if node.get("uncertain") is True or node.get("spool_terminal") is False:
        return True
    # a terminal failure counts as settled only once the generation failure has been validated
    if node.get("state") == "terminal_failure_received" and node.get("generation_failure") != "validated":
        return True
    words = (str(node.get(key, "")).lower() for key in ("state", "delivery_state"))
    return any("unknown" in w or "uncertain" in w for w in words)


def request_uncertain(state: Mapping[str, Any] | None) -> bool:
    """True when any level of a (nested) request-state record says the remote outcome is unknown."""
    pending = deque([state] if state else [])
    while pending:
        node = pending.popleft()
        if _node_uncertain(node):
            return True
        pending.extend(v for v in node.values() if isinstance(v, Mapping) and v)
    return False


__all__ = ["BENCHMARKS", "CancellationToken", "DatasetAdapter", "EpisodeBackend", "EpisodeIdentity", "EpisodePlan",
           "EpisodeResult", "ResourceRequirements", "SCHEMA_VERSION", "TaskSpec", "request_uncertain"]
