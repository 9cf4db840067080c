"""Check a (multi-node) process group before loading any weights: rank census by host, a checksum
all-reduce and the all-reduce bandwidth. The role of ``tests/distributed_nccl_smoke.py`` of the
reference; it is launched the same way as the training drivers:

    torchrun --nnodes 2 --nproc-per-node 8 ... -m tiny_dsv41_b200.parallel.smoke \
        --expected-nodes 2 --expected-local-world-size 8

Rank 0 prints one JSON line (hosts and their rank counts, the checksum, algorithm and bus
bandwidth of an all-reduce of ``--elements`` fp32 values, max time over ranks) and the run fails
when the census or the checksum is wrong. On CUDA the collective is timed with events on the
current stream; on CPU (gloo) with the host clock.
"""

from __future__ import annotations

import argparse
import json
import os
import socket
import time

import torch
import torch.distributed as dist


def parse_args(argv=None) -> argparse.Namespace:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--expected-nodes", type=int, default=None, help="fail unless the ranks span this many hosts")
    p.add_argument("--expected-local-world-size", type=int, default=None, help="ranks per host")
    p.add_argument("--elements", type=int, default=16 * 1024 * 1024, help="fp32 values per all-reduce")
    p.add_argument("--warmup", type=int, default=2)
    p.add_argument("--iterations", type=int, default=5)
    return p.parse_args(argv)


def host_census() -> dict[str, int]:
    names: list[str | None] = [None] * dist.get_world_size()
    dist.all_gather_object(names, socket.gethostname())
    return {host: names.count(host) for host in sorted(set(names))}


def checksum(device) -> tuple[float, float]:
    """Each rank adds rank + 1; the exact expected total is world (world + 1) / 2."""
    world = dist.get_world_size()
    value = torch.full((1,), float(dist.get_rank() + 1), dtype=torch.float64, device=device)
    dist.all_reduce(value)
    return value.item(), world * (world + 1) / 2


def allreduce_bandwidth(device, elements: int, warmup: int, iterations: int) -> dict:
    world = dist.get_world_size()
    buf = torch.ones(elements, dtype=torch.float32, device=device)
    for _ in range(warmup):
        dist.all_reduce(buf)
    if device.type == "cuda":
        torch.cuda.synchronize(device)
        dist.barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(iterations):
            dist.all_reduce(buf)
        end.record()
        torch.cuda.synchronize(device)
        seconds = start.elapsed_time(end) / 1e3 / iterations
    else:
        dist.barrier()
        t0 = time.perf_counter()
        for _ in range(iterations):
            dist.all_reduce(buf)
        seconds = (time.perf_counter() - t0) / iterations
    slowest = torch.tensor([seconds], dtype=torch.float64, device=device)
    dist.all_reduce(slowest, op=dist.ReduceOp.MAX)
    seconds = slowest.item()
    nbytes = elements * 4
    algbw = nbytes / seconds / 1e9
    return {"bytes": nbytes, "seconds": seconds, "algbw_gbs": algbw,
            "busbw_gbs": algbw * 2 * (world - 1) / world if world > 1 else algbw}


def run(args, device) -> dict:
    census = host_census()
    total, expected = checksum(device)
    report = {"world_size": dist.get_world_size(), "backend": dist.get_backend(), "hosts": census,
              "checksum": total, "checksum_expected": expected}
    errors = []
    if total != expected:
        errors.append(f"checksum {total} != {expected}")
    if args.expected_nodes is not None and len(census) != args.expected_nodes:
        errors.append(f"expected {args.expected_nodes} hosts, found {len(census)}: {census}")
    if args.expected_local_world_size is not None and any(n != args.expected_local_world_size
                                                          for n in census.values()):
        errors.append(f"expected {args.expected_local_world_size} ranks per host: {census}")
    if not errors:
        report["allreduce"] = allreduce_bandwidth(device, args.elements, args.warmup, args.iterations)
    report["ok"] = not errors
    report["errors"] = errors
    return report


def main(argv=None) -> None:
    from ..runtime import initialize_runtime

    args = parse_args(argv)
    runtime = initialize_runtime(require_distributed=True)
    try:
        report = run(args, runtime.device)
        if runtime.is_main:
            print(json.dumps(report, sort_keys=True), flush=True)
        if not report["ok"]:
            raise SystemExit(1)
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
