"""Per-kernel device time of one call, from the CUDA activity records of ``torch.profiler``.

Used by the benchmarks on an extra, untimed step: which kernels ran, how many times, and their
summed device time (each kernel's own duration, so concurrent streams are not double-counted as
wall time). ``own`` counts the kernels of this library (their names carry the ``tdsv``
namespace); ``other`` everything else (PyTorch elementwise kernels, NCCL, copies, memsets).
"""

from __future__ import annotations

import json

import torch


def kernel_census(fn, sync: bool = True) -> dict:
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        if sync:
            torch.cuda.synchronize()
    own = other = 0
    per_kernel: dict[str, list[float]] = {}
    for evt in prof.events():
        if evt.device_type != torch.autograd.DeviceType.CUDA:
            continue
        if "tdsv" in evt.name:
            own += 1
        else:
            other += 1
        entry = per_kernel.setdefault(evt.name[:160], [0, 0.0])
        entry[0] += 1
        entry[1] += evt.device_time
    rows = sorted(per_kernel.items(), key=lambda kv: -kv[1][1])
    total = sum(v[1] for _, v in rows)
    return {"own": own, "other": other, "total_kernel_us": total,
            "kernels": [{"name": n, "launches": c, "us": round(us, 1), "share": round(us / max(total, 1e-9), 4)}
                        for n, (c, us) in rows]}


def write_census(census: dict, path: str, **extra) -> None:
    with open(path, "w") as f:
        json.dump({**extra, **census}, f, indent=1)


__all__ = ["kernel_census", "write_census"]
