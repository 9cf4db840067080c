"""``train_qwen.py``: Qwen3-MoE training from HF safetensors with context, expert and FSDP2
parallelism on random token batches (the reference's ``train_qwen.py`` flags and summary).

Each step: random ids (first = BOS) from a per-data-rank generator, loss with the router
load-balancing term, backward, expert-gradient scaling, global-norm clipping at 1.0, AdamW.
The run fails if the tracked first-layer query weight did not change. The summary line
(``{"summary": {...}}``) reports sizes, last loss / aux loss / grad norm, timings and peak memory.
"""

from __future__ import annotations

import argparse
import json
import time
from pathlib import Path

import torch
import torch.distributed as dist

from ..ops import StatusMonitor
from ..models.qwen import Qwen3MoeConfig, load_qwen3_moe
from ..parallel.cp import ContextParallel
from ..parallel.dispatch import TokenDispatcher
from ..parallel.fsdp import apply_fsdp, clip_grad_norm_, expert_parameters, scale_expert_grads
from ..runtime import distributed_mean, initialize_runtime, local_tensor
from ..utils.trace import trace_point


def parse_args(argv=None):
    p = argparse.ArgumentParser(description="Train Qwen3-MoE with CP, EP and FSDP2")
    p.add_argument("--model-path", required=True)
    p.add_argument("--steps", type=int, default=1)
    p.add_argument("--batch-size", type=int, default=1)
    p.add_argument("--seq-len", type=int, default=16)
    p.add_argument("--learning-rate", type=float, default=1e-4)
    p.add_argument("--seed", type=int, default=42)
    p.add_argument("--cp-size", type=int, default=1)
    p.add_argument("--ep-size", type=int, default=1)
    p.add_argument("--metrics-file")
    p.add_argument("--gradient-checkpointing", action="store_true")
    p.add_argument("--device", default="auto")
    return p.parse_args(argv)


def validate_args(args) -> None:
    if args.steps < 1 or args.batch_size < 1:
        raise ValueError("steps and batch-size must be positive")
    if args.seq_len < 2:
        raise ValueError("seq-len must be at least 2")
    if args.learning_rate <= 0:
        raise ValueError("learning-rate must be positive")
    if args.cp_size < 1 or args.ep_size < 1:
        raise ValueError("cp-size and ep-size must be positive")
    if args.seq_len % args.cp_size:
        raise ValueError("seq-len must divide evenly across cp-size")
    if not Path(args.model_path).is_dir():
        raise FileNotFoundError(f"model path does not exist: {args.model_path}")


def build(args, runtime):
    meshes, cp, dispatcher = None, ContextParallel(), TokenDispatcher()
    if runtime.distributed and runtime.world_size > 1:
        from ..parallel.meshes import ParallelMeshes

        meshes = ParallelMeshes.build(cp=args.cp_size, ep=args.ep_size, device_type=runtime.device.type)
        cp = ContextParallel(meshes.cp)
        if meshes.ep is not None:
            if runtime.device.type == "cuda":
                from ..parallel.nvlink_ep import NVLinkTokenDispatcher

                dispatcher = NVLinkTokenDispatcher(meshes.ep, max_tokens=args.batch_size * args.seq_len // args.cp_size)
            else:
                from ..parallel.dispatch import AllToAllTokenDispatcher

                dispatcher = AllToAllTokenDispatcher(meshes.ep)
    dtype = torch.bfloat16 if runtime.device.type == "cuda" else torch.float32
    model = load_qwen3_moe(args.model_path, device=runtime.device, dtype=dtype, context_parallel=cp,
                           token_dispatcher=dispatcher)
    return model, meshes, cp


def train(args, runtime) -> dict:
    torch.manual_seed(args.seed)
    started = time.perf_counter()
    model, meshes, cp = build(args, runtime)
    loaded = time.perf_counter()
    if args.gradient_checkpointing:
        model.gradient_checkpointing_enable()
    model.train()
    experts = sum(p.numel() for p in expert_parameters(model))
    dense = sum(p.numel() for p in model.parameters()) - experts
    full_count = dense + experts * args.ep_size
    if meshes is not None:
        apply_fsdp(model, meshes, param_dtype=next(model.parameters()).dtype)
    sharded = time.perf_counter()
    optimizer = torch.optim.AdamW(model.parameters(), lr=args.learning_rate, foreach=False)
    data_rank = runtime.rank // args.cp_size
    generator = torch.Generator(device=runtime.device)
    generator.manual_seed(args.seed + data_rank)
    tracked = model.model.layers[0].self_attn.q_proj.weight
    before = local_tensor(tracked).detach().float().clone()
    loss_v = aux_v = norm_v = 0.0
    monitor = StatusMonitor(runtime.device)
    for step in range(1, args.steps + 1):
        trace_point("step_begin", step=step)
        ids = torch.randint(0, model.config.vocab_size, (args.batch_size, args.seq_len), device=runtime.device,
                            generator=generator)
        ids[:, 0] = model.config.bos_token_id
        optimizer.zero_grad(set_to_none=True)
        out = model(ids, labels=ids, output_router_logits=True)
        if out.loss is None or not torch.isfinite(out.loss):
            raise RuntimeError("training produced a non-finite loss")
        out.loss.backward()
        scale_expert_grads(model, args.ep_size)
        norm = clip_grad_norm_(list(model.parameters()), 1.0)
        optimizer.step()
        loss_v = distributed_mean(out.loss, runtime)
        if isinstance(out.aux_loss, torch.Tensor):
            aux_v = distributed_mean(out.aux_loss, runtime)
        norm_v = float(norm)
        monitor.step_end(f"step {step}")
        trace_point("step_end", step=step, loss=loss_v, grad_norm=norm_v)
        if runtime.is_main:
            print(json.dumps({"step": step, "loss": loss_v, "aux_loss": aux_v, "grad_norm": norm_v}), flush=True)
    delta = (local_tensor(tracked).detach().float() - before).abs().max()
    if dist.is_initialized():
        dist.all_reduce(delta, op=dist.ReduceOp.MAX)
    if delta.item() == 0:
        raise RuntimeError("optimizer step did not update the tracked parameter")
    if runtime.device.type == "cuda":
        torch.cuda.synchronize(runtime.device)
    finished = time.perf_counter()
    world = runtime.world_size
    metrics = {"model": "Qwen3-MoE", "parameters": full_count, "world_size": world, "cp_size": args.cp_size,
               "ep_size": args.ep_size, "fsdp_size": world, "expert_fsdp_size": world // args.ep_size,
               "steps": args.steps, "batch_size_per_data_rank": args.batch_size,
               "global_batch_size": args.batch_size * (world // args.cp_size), "sequence_length": args.seq_len,
               "loss": loss_v, "aux_loss": aux_v, "grad_norm": norm_v, "parameter_delta_max": delta.item(),
               "load_seconds": loaded - started, "shard_seconds": sharded - loaded, "train_seconds": finished - sharded,
               "peak_memory_gib": (torch.cuda.max_memory_allocated(runtime.device) / 2 ** 30
                                   if runtime.device.type == "cuda" else 0.0)}
    if runtime.is_main:
        print(json.dumps({"summary": metrics}), flush=True)
        if args.metrics_file:
            path = Path(args.metrics_file)
            path.parent.mkdir(parents=True, exist_ok=True)
            path.write_text(json.dumps(metrics, indent=2) + "\n", encoding="utf-8")
    return metrics


def main(argv=None) -> None:
    args = parse_args(argv)
    validate_args(args)
    runtime = None
    try:
        runtime = initialize_runtime(args.device, require_distributed=True)
        train(args, runtime)
    finally:
        if runtime is not None and dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
