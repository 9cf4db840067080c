"""Low-frequency host, cgroup and GPU counters for rollout runs (``rollout_manager/telemetry.py:24-100``).

``snapshot`` reads /proc and cgroup v2 counters and one ``nvidia-smi`` query (never changes any
setting); ``process_accounting`` walks the owned process tree; ``monitor`` appends one JSON sample
per interval to a (optionally gzip) file with a size ceiling.
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

_PROC = {"stat": "/proc/stat", "memory": "/proc/meminfo", "load": "/proc/loadavg", "netdev": "/proc/net/dev",
         "cpu_pressure": "/proc/pressure/cpu", "memory_pressure": "/proc/pressure/memory",
         "io_pressure": "/proc/pressure/io", "cgroup_cpu": "/sys/fs/cgroup/cpu.stat",
         "cgroup_cpu_max": "/sys/fs/cgroup/cpu.max", "cgroup_memory": "/sys/fs/cgroup/memory.current",
         "cgroup_memory_max": "/sys/fs/cgroup/memory.max", "cgroup_io": "/sys/fs/cgroup/io.stat"}
GPU_FIELDS = "index,uuid,utilization.gpu,utilization.memory,memory.used,power.draw,clocks.sm,clocks.mem,temperature.gpu"


def _read(path):
    try:
        return Path(path).read_text()
    except OSError as exc:
        return {"unavailable": type(exc).__name__}


def snapshot() -> dict:
    start = time.monotonic()
    out = {"unix_ns": time.time_ns(), "monotonic_ns": time.monotonic_ns(), "host": socket.gethostname(),
           "cpu_affinity": sorted(os.sched_getaffinity(0))}
    out.update({k: _read(p) for k, p in _PROC.items()})
    try:
        out["gpu_fields"] = GPU_FIELDS.split(",")
        out["gpu_csv"] = subprocess.check_output(["nvidia-smi", "--query-gpu=" + GPU_FIELDS,
                                                  "--format=csv,noheader,nounits"], text=True, timeout=3).strip()
    except (OSError, subprocess.SubprocessError) as exc:
        out["gpu_error"] = str(exc)
    out["disk_free_bytes"] = shutil.disk_usage(".").free
    out["sample_seconds"] = time.monotonic() - start
    return out


def process_accounting(root_pid: int) -> dict:
    pending, seen, rows = [root_pid], set(), []
    while pending and len(seen) < 4096:
        pid = pending.pop()
        if pid in seen:
            continue
        seen.add(pid)
        root = Path("/proc") / str(pid)
        try:
            stat = (root / "stat").read_text().rsplit(")", 1)[1].split()
            status = dict(line.split(":", 1) for line in (root / "status").read_text().splitlines() if ":" in line)
            for task in (root / "task").iterdir():
                try:
                    pending.extend(map(int, (task / "children").read_text().split()))
                except OSError:
                    pass
            rows.append({"pid": pid, "user_ticks": int(stat[11]), "system_ticks": int(stat[12]),
                         "minor_faults": int(stat[7]), "major_faults": int(stat[9]),
                         "status": {k: status.get(k, "").strip() for k in ("Name", "VmRSS", "RssAnon", "Threads")}})
        except (OSError, IndexError, ValueError):
            pass
    return {"clock_ticks_per_second": os.sysconf("SC_CLK_TCK"), "processes": rows, "truncated": bool(pending)}


def monitor(path, stop: threading.Event, *, interval: float = 2, ttl: float = 21600, extra=None) -> None:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    end = time.monotonic() + ttl
    opener = gzip.open if path.suffix == ".gz" else open
    limit = (1536 if path.suffix == ".gz" else 512) << 20
    with opener(path, "xt") as out:
        while not stop.is_set() and time.monotonic() < end:
            t0 = time.monotonic()
            sample = snapshot()
            if extra is not None:
                sample["manager"] = extra()
                sample["owned_process_accounting"] = process_accounting(os.getpid())
            out.write(json.dumps(sample) + "\n")
            out.flush()
            if out.tell() > limit:
                raise RuntimeError("telemetry exceeded its size ceiling")
            stop.wait(max(0.0, interval - (time.monotonic() - t0)))


__all__ = ["monitor", "process_accounting", "snapshot"]
