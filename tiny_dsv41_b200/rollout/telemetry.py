"""Low-frequency host, cgroup and GPU counters for rollout runs.

Sample content follows ``rollout_manager/telemetry.py:24-100`` (the analysis tools read these
files): raw text of the /proc and cgroup-v2 counter files, one ``nvidia-smi`` query of read-only
fields (no setting is ever changed), free disk space and how long the sample took. The
per-process accounting walks the process tree owned by the manager. ``monitor`` appends one JSON
line per interval to a plain or gzip file and stops at a size ceiling.
"""

from __future__ import annotations

import gzip
import json
import os
import shutil
import socket
import subprocess
import threading
import time
from pathlib import Path

COUNTER_FILES = (
    ("stat", "/proc/stat"), ("memory", "/proc/meminfo"), ("load", "/proc/loadavg"), ("netdev", "/proc/net/dev"),
    ("cpu_pressure", "/proc/pressure/cpu"), ("memory_pressure", "/proc/pressure/memory"),
    ("io_pressure", "/proc/pressure/io"), ("cgroup_cpu", "/sys/fs/cgroup/cpu.stat"),
    ("cgroup_cpu_max", "/sys/fs/cgroup/cpu.max"), ("cgroup_memory", "/sys/fs/cgroup/memory.current"),
    ("cgroup_memory_max", "/sys/fs/cgroup/memory.max"), ("cgroup_io", "/sys/fs/cgroup/io.stat"),
)
GPU_FIELDS = "index,uuid,utilization.gpu,utilization.memory,memory.used,power.draw,clocks.sm,clocks.mem,temperature.gpu"
MAX_PROCESSES = 4096


def _counter(path: str):
    try:
        return Path(path).read_text()
    except OSError as error:
        return {"unavailable": type(error).__name__}


def _gpu_query() -> dict:
    try:
        csv = subprocess.check_output(["nvidia-smi", f"--query-gpu={GPU_FIELDS}", "--format=csv,noheader,nounits"],
                                      text=True, timeout=3)
    except (OSError, subprocess.SubprocessError) as error:
        return {"gpu_error": str(error)}
    return {"gpu_fields": GPU_FIELDS.split(","), "gpu_csv": csv.strip()}


def snapshot() -> dict:
    began = time.monotonic()
    sample = {"unix_ns": time.time_ns(), "monotonic_ns": time.monotonic_ns(), "host": socket.gethostname(),
              "cpu_affinity": sorted(os.sched_getaffinity(0))}
    for key, path in COUNTER_FILES:
        sample[key] = _counter(path)
    sample.update(_gpu_query())
    sample["disk_free_bytes"] = shutil.disk_usage(".").free
    sample["sample_seconds"] = time.monotonic() - began
    return sample


def _process_row(pid: int) -> tuple[dict, list[int]]:
    """(accounting row, child pids) of one process; raises OSError / ValueError if it vanished."""
    proc = Path("/proc") / str(pid)
    fields = (proc / "stat").read_text().rsplit(")", 1)[1].split()  # after the command name
    status = {}
    for line in (proc / "status").read_text().splitlines():
        name, colon, value = line.partition(":")
        if colon:
            status[name] = value.strip()
    children = []
    for task in (proc / "task").iterdir():
        try:
            children += [int(c) for c in (task / "children").read_text().split()]
        except OSError:
            continue
    row = {"pid": pid, "user_ticks": int(fields[11]), "system_ticks": int(fields[12]),
           "minor_faults": int(fields[7]), "major_faults": int(fields[9]),
           "status": {key: status.get(key, "") for key in ("Name", "VmRSS", "RssAnon", "Threads")}}
    return row, children


def process_accounting(root_pid: int) -> dict:
    stack, visited, rows = [root_pid], set(), []
    while stack and len(visited) < MAX_PROCESSES:
        pid = stack.pop()
        if pid in visited:
            continue
        visited.add(pid)
        try:
            row, children = _process_row(pid)
        except (OSError, IndexError, ValueError):
            continue
        rows.append(row)
        stack.extend(children)
    return {"clock_ticks_per_second": os.sysconf("SC_CLK_TCK"), "processes": rows, "truncated": bool(stack)}


def monitor(path, stop: threading.Event, *, interval: float = 2, ttl: float = 21600, extra=None) -> None:
    """Write samples every `interval` seconds until `stop` is set or `ttl` seconds have passed;
    ``extra()`` adds the manager's own state and the owned process tree to each sample."""
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    compressed = path.suffix == ".gz"
    ceiling = (1536 if compressed else 512) * 2 ** 20
    deadline = time.monotonic() + ttl
    with (gzip.open if compressed else open)(path, "xt") as sink:
        while not stop.is_set() and time.monotonic() < deadline:
            began = time.monotonic()
            sample = snapshot()
            if extra is not None:
                sample["manager"] = extra()
                sample["owned_process_accounting"] = process_accounting(os.getpid())
            sink.write(json.dumps(sample) + "\n")
            sink.flush()
            if sink.tell() > ceiling:
                raise RuntimeError("telemetry exceeded its size ceiling")
            stop.wait(max(0.0, interval - (time.monotonic() - began)))


__all__ = ["monitor", "process_accounting", "snapshot"]
