"""Child process: bench_ep.py's reference expert arms on CPU gloo ranks (one step each)."""

import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench_ep  # noqa: E402

dist.init_process_group("gloo")
rank, world = dist.get_rank(), dist.get_world_size()
from torch.distributed.device_mesh import init_device_mesh  # noqa: E402

mesh = init_device_mesh("cpu", (world,), mesh_dim_names=("ep",))
for arm in ("dsv4", "qwen"):
    args = bench_ep.parse_args(["--impl", "reference", "--tokens", "64", "--hidden", "64", "--experts", "8",
                                "--topk", "2", "--intermediate", "32", "--reference-experts", arm])
    tensors = bench_ep._inputs(args, rank, world, torch.device("cpu"))
    step = bench_ep._reference_step(args, mesh, tensors, True)
    step()
    print(f"rank {rank} arm {arm} ok", flush=True)
dist.barrier()
dist.destroy_process_group()
