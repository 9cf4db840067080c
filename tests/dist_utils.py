"""Run a function on N gloo CPU ranks (torch.multiprocessing spawn, file:// rendezvous)."""

import os
import tempfile
import traceback

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _entry(rank, world, init_file, fn, args, errors):
    try:
        dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
        fn(rank, world, *args)
    except Exception:  # pragma: no cover - reported to the parent
        errors.put((rank, traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def run_gloo(fn, world: int = 2, *args):
    ctx = mp.get_context("spawn")
    errors = ctx.SimpleQueue()
    with tempfile.TemporaryDirectory() as tmp:
        init_file = os.path.join(tmp, "rendezvous")
        procs = [ctx.Process(target=_entry, args=(r, world, init_file, fn, args, errors)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=300)
        messages = []
        while not errors.empty():
            messages.append(errors.get())
        for p in procs:
            if p.is_alive():
                p.kill()
                messages.append((-1, "rank timed out"))
            elif p.exitcode not in (0, None):
                messages.append((-1, f"exit code {p.exitcode}"))
        if messages:
            raise AssertionError("\n".join(f"rank {r}: {m}" for r, m in messages))
