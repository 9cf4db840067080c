"""Host-side stage intervals as JSON lines with an explicit clock domain
(``rollout_manager/analysis/stage_timings.py`` format: one record per interval with name,
start/end/duration seconds, clock domain and details)."""

from __future__ import annotations

import json
import os
import time
from contextlib import contextmanager
from pathlib import Path


class StageTimings:
    def __init__(self, path, *, clock_domain: str = "process_monotonic") -> None:
        self.path = Path(path)
        self.path.parent.mkdir(parents=True, exist_ok=True)
        self.clock_domain = clock_domain

    def _write(self, record: dict) -> None:
        with self.path.open("a", encoding="utf-8") as f:
            f.write(json.dumps(record, sort_keys=True, allow_nan=False) + "\n")

    @contextmanager
    def interval(self, name: str, **details):
        start = time.monotonic()
        try:
            yield
        finally:
            end = time.monotonic()
            self._write({"stage": name, "start": start, "end": end, "seconds": end - start,
                         "clock_domain": self.clock_domain, "pid": os.getpid(), "details": details})

    def call(self, name: str, fn, *args, details: dict | None = None, **kwargs):
        with self.interval(name, **(details or {})):
            return fn(*args, **kwargs)


__all__ = ["StageTimings"]
