"""Opt-in tracing: per-rank JSON trace points and NVTX ranges.

* ``TDSV_DISTRIBUTED_TRACE=1`` makes ``trace_point(event, **fields)`` print one JSON line per call to
  stderr with the rank, local rank, host-monotonic and wall time (the role of
  ``DSV41_DISTRIBUTED_TRACE`` in ``train_dsv4_checkpoint.py:29-31, 198-222`` of the reference). A
  path in ``TDSV_DISTRIBUTED_TRACE_DIR`` writes ``trace-rank-R.jsonl`` files there instead.
* ``TDSV_NVTX=1`` turns ``nvtx_range(name)`` into a ``torch.cuda.nvtx`` push / pop pair, so a
  timeline profiler shows the framework's phases (attention, MoE, EP dispatch / combine);
  otherwise it costs one flag test.
"""

from __future__ import annotations

import json
import os
import sys
import time
from contextlib import contextmanager

_TRACE = os.environ.get("TDSV_DISTRIBUTED_TRACE", "") not in ("", "0")
_TRACE_DIR = os.environ.get("TDSV_DISTRIBUTED_TRACE_DIR") or None
_NVTX = os.environ.get("TDSV_NVTX", "") not in ("", "0")


def tracing_enabled() -> bool:
    return _TRACE or bool(_TRACE_DIR)


def trace_point(event: str, **fields) -> None:
    if not tracing_enabled():
        return
    record = {"event": event, "rank": int(os.environ.get("RANK", "0")),
              "local_rank": int(os.environ.get("LOCAL_RANK", "0")), "monotonic": time.monotonic(),
              "time": time.time(), "pid": os.getpid(), **fields}
    line = json.dumps(record, sort_keys=True, default=str)
    if _TRACE_DIR:
        os.makedirs(_TRACE_DIR, exist_ok=True)
        with open(os.path.join(_TRACE_DIR, f"trace-rank-{record['rank']}.jsonl"), "a", encoding="utf-8") as f:
            f.write(line + "\n")
    else:
        print(line, file=sys.stderr, flush=True)


@contextmanager
def nvtx_range(name: str):
    if not _NVTX:
        yield
        return
    import torch

    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


def set_tracing(*, distributed: bool | None = None, nvtx: bool | None = None, directory: str | None = None) -> None:
    """Programmatic switch (tests, notebooks); the environment variables set the defaults."""
    global _TRACE, _NVTX, _TRACE_DIR
    if distributed is not None:
        _TRACE = distributed
    if nvtx is not None:
        _NVTX = nvtx
    if directory is not None:
        _TRACE_DIR = directory or None


__all__ = ["nvtx_range", "set_tracing", "trace_point", "tracing_enabled"]
