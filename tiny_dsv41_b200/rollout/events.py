"""Append-only event log and immutable result files of one rollout run.

Record fields are the interface of ``rollout_manager/events.py:28-76`` (the learner and the
rollout service read each other's runs):

* ``events.jsonl``: one JSON line per event, numbered by a per-run sequence, stamped with both
  the wall clock (``unix_ns``) and the coordinator's monotonic clock;
* ``results/<sha256 of the canonical identity JSON>.json`` and ``summary.json``: created
  exclusively and fsynced, so a written result can never be replaced.
"""

from __future__ import annotations

import dataclasses
import hashlib
import json
import os
import threading
import time
from itertools import count
from pathlib import Path
from typing import Any, Mapping

from .contracts import SCHEMA_VERSION

CLOCK_DOMAIN = "coordinator_monotonic"


def json_value(value: Any) -> Any:
    """Plain JSON data for dataclasses, mappings, sequences and paths (recursively)."""
    if dataclasses.is_dataclass(value) and not isinstance(value, type):
        return {f.name: json_value(getattr(value, f.name)) for f in dataclasses.fields(value)}
    if isinstance(value, Mapping):
        return {str(key): json_value(item) for key, item in value.items()}
    if isinstance(value, (list, tuple)):
        return list(map(json_value, value))
    return str(value) if isinstance(value, Path) else value


def identity_key(identity: Any) -> str:
    canonical = json.dumps(json_value(identity), sort_keys=True, separators=(",", ":"))
    return hashlib.sha256(canonical.encode()).hexdigest()


def _write_exclusive(path: Path, value: Any) -> Path:
    """Create `path` (never overwrite), write `value` as indented JSON and fsync it."""
    with path.open("x", encoding="utf-8") as handle:
        handle.write(json.dumps(json_value(value), indent=2, allow_nan=False) + "\n")
        handle.flush()
        os.fsync(handle.fileno())
    return path


class EventStore:
    """Owns ``root`` (created here; an existing directory is an error)."""

    def __init__(self, root, run_id: str) -> None:
        self.root, self.run_id = Path(root), run_id
        self.root.parent.mkdir(parents=True, exist_ok=True)
        self.root.mkdir(exist_ok=False)
        (self.root / "results").mkdir()
        self._lock = threading.Lock()
        self._numbers = count()
        self._log = (self.root / "events.jsonl").open("x", encoding="utf-8")
        self.append("run_created")

    def append(self, event: str, identity=None, *, turn_id=None, request_id=None, tool_call_id=None, trial_id=None,
               **details) -> dict:
        who = json_value(identity)
        if trial_id is None and isinstance(who, dict):
            trial_id = who.get("trial_id")
        record = {
            "schema_version": SCHEMA_VERSION, "run_id": self.run_id, "clock_domain": CLOCK_DOMAIN,
            "unix_ns": time.time_ns(), "monotonic_ns": time.monotonic_ns(), "event": event, "identity": who,
            "turn_id": turn_id, "request_id": request_id, "tool_call_id": tool_call_id, "trial_id": trial_id,
            "details": json_value(details),
        }
        with self._lock:  # sequence numbers follow the order of the lines in the file
            record["sequence"] = next(self._numbers)
            self._log.write(json.dumps(record, allow_nan=False) + "\n")
            self._log.flush()
        return record

    def write_result(self, result) -> Path:
        body = {"schema_version": SCHEMA_VERSION, **json_value(result)}
        return _write_exclusive(self.root / "results" / f"{identity_key(result.identity)}.json", body)

    def write_summary(self, summary: Mapping[str, Any]) -> Path:
        body = {"schema_version": SCHEMA_VERSION, "run_id": self.run_id, **json_value(summary)}
        return _write_exclusive(self.root / "summary.json", body)

    def close(self) -> None:
        with self._lock:
            self._log.close()


__all__ = ["EventStore", "identity_key", "json_value"]
