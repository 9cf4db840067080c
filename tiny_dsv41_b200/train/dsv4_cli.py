"""``train_dsv4_checkpoint.py``: train a window of layers of a released DeepSeek-V4.1 checkpoint
(FP8 / FP4 weights dequantised on load) with expert, context and FSDP2 parallelism on random
tokens - the reference's ``train_dsv4_checkpoint.py`` flags, checks and summary.

SGD or AdamW; ``--optimizer-in-backward`` applies SGD from post-accumulate-grad hooks on bf16
shards with the backward scaled by 2^-16 (the learning rate is divided by the same power of
two, so the update is unchanged while bf16 gradients keep their range); a non-finite update on
any rank aborts the run. ``--sequence-packing`` packs the batch into one stream with sequence
ids so attention and the Engram hash stop at sequence boundaries.
"""

from __future__ import annotations

import argparse
import json
import time
from pathlib import Path

import torch
import torch.distributed as dist

from ..ops import StatusMonitor
from ..models.dsv4 import DeepSeekV41Config
from ..parallel.cp import ContextParallel, pack_sequences
from ..parallel.dispatch import TokenDispatcher
from ..parallel.fsdp import apply_fsdp, expert_parameters, scale_expert_grads
from ..runtime import distributed_mean, initialize_runtime, local_tensor
from ..utils.trace import trace_point

IN_BACKWARD_SCALE = 2.0 ** -16


def parse_args(argv=None):
    p = argparse.ArgumentParser(description="Train a window of a released DeepSeek-V4.1 checkpoint")
    p.add_argument("--model-path", required=True)
    p.add_argument("--steps", type=int, default=1)
    p.add_argument("--start-layer", type=int, default=0)
    p.add_argument("--num-layers", type=int, default=1)
    p.add_argument("--batch-size", type=int, default=1)
    p.add_argument("--seq-len", type=int, default=8)
    p.add_argument("--learning-rate", type=float, default=1e-4)
    p.add_argument("--optimizer", choices=("sgd", "adamw"), default="sgd")
    p.add_argument("--cp-size", type=int, default=1)
    p.add_argument("--ep-size", type=int, default=8)
    p.add_argument("--seed", type=int, default=42)
    p.add_argument("--metrics-file")
    p.add_argument("--gradient-checkpointing", action="store_true")
    p.add_argument("--optimizer-in-backward", action="store_true")
    p.add_argument("--sequence-packing", action="store_true")
    p.add_argument("--device", default="auto")
    return p.parse_args(argv)


def validate_args(args, world_size: int) -> None:
    root = Path(args.model_path)
    if not root.is_dir():
        raise FileNotFoundError(f"model path does not exist: {root}")
    for name in ("config.json", "model.safetensors.index.json"):
        if not (root / name).is_file():
            raise FileNotFoundError(f"checkpoint file does not exist: {root / name}")
    if args.steps < 1 or args.batch_size < 1 or args.num_layers < 1 or args.seq_len < 2:
        raise ValueError("steps, batch-size, and num-layers must be positive; seq-len must be at least 2")
    if args.start_layer < 0:
        raise ValueError("start-layer must be non-negative")
    if args.learning_rate <= 0:
        raise ValueError("learning-rate must be positive")
    if args.cp_size < 1 or args.ep_size < 1 or world_size % args.cp_size or world_size % args.ep_size:
        raise ValueError("cp-size and ep-size must both divide world size")
    length = args.seq_len * args.batch_size if args.sequence_packing else args.seq_len
    if length % args.cp_size:
        raise ValueError("sequence length after packing must divide evenly across cp-size")
    config = DeepSeekV41Config.from_json(root / "config.json")
    if config.n_routed_experts % args.ep_size:
        raise ValueError("the configured n_routed_experts must divide evenly across ep-size")
    if args.optimizer_in_backward and args.optimizer != "sgd":
        raise ValueError("optimizer-in-backward requires SGD")


def train(args, runtime) -> dict:
    from ..models.dsv4.checkpoint import load_dsv41_backbone_window

    validate_args(args, runtime.world_size)
    torch.manual_seed(args.seed)
    meshes, cp, dispatcher = None, ContextParallel(), TokenDispatcher()
    if runtime.world_size > 1:
        from ..parallel.meshes import ParallelMeshes

        meshes = ParallelMeshes.build(cp=args.cp_size, ep=args.ep_size, device_type=runtime.device.type, engram=True)
        cp = ContextParallel(meshes.cp)
        if meshes.ep is not None:
            if runtime.device.type == "cuda":
                from ..parallel.nvlink_ep import NVLinkTokenDispatcher

                length = args.seq_len * args.batch_size
                dispatcher = NVLinkTokenDispatcher(meshes.ep, max_tokens=length // args.cp_size)
            else:
                from ..parallel.dispatch import AllToAllTokenDispatcher

                dispatcher = AllToAllTokenDispatcher(meshes.ep)
    dtype = torch.bfloat16 if runtime.device.type == "cuda" else torch.float32
    started = time.perf_counter()
    model = load_dsv41_backbone_window(
        args.model_path, start_layer=args.start_layer, num_layers=args.num_layers, device=runtime.device,
        dtype=dtype, context_parallel=cp, token_dispatcher=dispatcher,
        engram_mesh=meshes.engram if meshes is not None else None, sparse_engram_gradients=args.optimizer == "sgd")
    if args.gradient_checkpointing:
        model.gradient_checkpointing_enable()
    model.train()
    loaded = time.perf_counter()
    trace_point("loaded", seconds=loaded - started)
    experts = sum(p.numel() for p in expert_parameters(model))
    tables = list(model.model.engram_tables.values())
    local_engram = sum(t.weight.numel() for t in tables)
    global_engram = sum(t.global_num_embeddings * model.config.engram_head_dim for t in tables)
    local_count = sum(p.numel() for p in model.parameters())
    full_count = local_count - experts - local_engram + experts * args.ep_size + global_engram
    if meshes is not None:
        apply_fsdp(model, meshes, param_dtype=dtype)
    sharded = time.perf_counter()
    trace_point("sharded", seconds=sharded - loaded)
    tracked = model.model.layers[0].attention_hc.fn
    before = local_tensor(tracked).detach().float().clone()
    scale = IN_BACKWARD_SCALE if args.optimizer_in_backward else 1.0
    lr = args.learning_rate / scale
    params = [p for p in model.parameters() if p.requires_grad]
    in_backward = None
    if args.optimizer_in_backward:
        from ..optim.sgd import install_sgd_in_backward

        in_backward = install_sgd_in_backward(params, lr, expert_divisor=float(args.ep_size),
                                              expert_params=expert_parameters(model))
        optimizer = None
    elif args.optimizer == "adamw":
        optimizer = torch.optim.AdamW(params, lr=lr, foreach=False)
    else:
        optimizer = torch.optim.SGD(params, lr=lr, foreach=False)
    generator = torch.Generator(device=runtime.device)
    generator.manual_seed(args.seed + runtime.rank // args.cp_size)
    loss_v = aux_v = 0.0
    monitor = StatusMonitor(runtime.device)
    for step in range(1, args.steps + 1):
        trace_point("step_begin", step=step)
        ids = torch.randint(3, model.config.vocab_size, (args.batch_size, args.seq_len), device=runtime.device,
                            generator=generator)
        ids[:, 0] = model.config.bos_token_id
        seq = None
        if args.sequence_packing:
            ids, seq = pack_sequences(ids)
        if optimizer is not None:
            optimizer.zero_grad(set_to_none=True)
        if in_backward is not None:
            in_backward.reset()
        out = model(ids, labels=ids, sequence_ids=seq)
        if out.loss is None or not torch.isfinite(out.loss):
            raise RuntimeError("training produced a non-finite loss")
        (out.loss * scale).backward()
        if in_backward is not None:
            finite = torch.tensor(int(in_backward.finite()), device=runtime.device, dtype=torch.int32)
            if dist.is_initialized():
                dist.all_reduce(finite, op=dist.ReduceOp.MIN)
            if not finite.item():
                raise RuntimeError("non-finite in-backward SGD update; abort and reload the checkpoint")
        else:
            scale_expert_grads(model, args.ep_size)
            optimizer.step()
        loss_v = distributed_mean(out.loss, runtime)
        aux_v = distributed_mean(out.aux_loss, runtime)
        monitor.step_end(f"step {step}")
        trace_point("step_end", step=step, loss=loss_v)
        if runtime.is_main:
            print(json.dumps({"step": step, "loss": loss_v, "aux_loss": aux_v}), flush=True)
    delta = (local_tensor(tracked).detach().float() - before).abs().max()
    if dist.is_initialized():
        dist.all_reduce(delta, op=dist.ReduceOp.MAX)
    if not torch.isfinite(delta):
        raise RuntimeError("optimizer step produced a non-finite parameter update")
    if delta.item() == 0:
        raise RuntimeError("optimizer step did not update the tracked parameter")
    if runtime.device.type == "cuda":
        torch.cuda.synchronize(runtime.device)
    finished = time.perf_counter()
    window = (f"DeepSeek-V4.1 {args.num_layers}-layer prefix" if args.start_layer == 0 else
              f"DeepSeek-V4.1 layers {args.start_layer}-{args.start_layer + args.num_layers - 1} window")
    metrics = {"model": window, "checkpoint": str(Path(args.model_path).resolve()), "parameters": full_count,
               "local_parameters_before_fsdp": local_count, "world_size": runtime.world_size,
               "cp_size": args.cp_size, "ep_size": args.ep_size, "fsdp_size": runtime.world_size,
               "experts_per_rank": model.model.layers[0].moe.routed.num_experts,
               "engram_rows_per_rank": sum(t.weight.shape[0] for t in tables),
               "sparse_engram_gradients": args.optimizer == "sgd", "steps": args.steps,
               "batch_size_per_rank": args.batch_size, "sequence_length": args.seq_len,
               "start_layer": args.start_layer, "optimizer": args.optimizer, "loss": loss_v, "aux_loss": aux_v,
               "parameter_delta_max": delta.item(), "load_seconds": loaded - started,
               "shard_seconds": sharded - loaded, "train_seconds": finished - sharded,
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
    runtime = None
    try:
        runtime = initialize_runtime(args.device, require_distributed=True)
        train(args, runtime)
    finally:
        if runtime is not None and dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
