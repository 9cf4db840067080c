"""DeepSeek-V4.1-Flash LoRA SFT benchmark: tokens/s for the whole job.

Flash dimensions (``tiny_dsv41_b200/models/dsv4/flash_config.json``: hidden 5120, 64 heads x 512,
window 128, sparse indexer top-512, 384 routed experts top-6 with intermediate 2304, mHC with 4
streams, two Engram tables), the first 40 layers, random-init weights (std 0.02). The routed
experts are frozen in the released MXFP4 layout (E2M1 codes + E8M0 scales per 32, random) and the
grouped GEMMs read them packed; EP = N over the experts; the Engram tables stay in host memory
(offload) with rows sharded over the ranks; LoRA rank 16 on the query projections (``q_a``,
``q_b``), AdamW on the adapters, gradient checkpointing. Data: seq 4096, batch 1 per rank,
uniform-random token ids, loss on every token.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 8 --master-addr 127.0.0.1 \\
        bench_dsv4.py --gpus 8
    python bench_dsv4.py --config tiny --layers 2 --seq-len 64 --device cpu   # plumbing check

The model is built in place (``models.dsv4.synthetic``) instead of loaded from a written
checkpoint: the 40-layer Flash prefix holds about 290 GB of FP4 experts. Rank 0 prints one JSON
line; the time brackets exactly ``--steps`` steps with a barrier and a device synchronisation on
both sides and is the max over ranks.
"""

from __future__ import annotations

import argparse
import json
import os
import time
from datetime import timedelta

ROOT = os.path.dirname(os.path.abspath(__file__))
METRIC = "SFT tokens/sec/box (max over ranks)"
CONFIGS = {"flash": os.path.join(ROOT, "tiny_dsv41_b200", "models", "dsv4", "flash_config.json"),
           "tiny": os.path.join(ROOT, "tiny_dsv41_b200", "models", "dsv4", "tiny_config.json")}
HBM_BYTES = 178 * 2 ** 30
ACTIVATION_RESERVE = 48 * 2 ** 30  # 40 checkpointed layers of 4 mHC streams, recompute transients, slabs


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--gpus", type=int, default=8)
    p.add_argument("--steps", type=int, default=3)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--config", default="flash", help="flash, tiny or a config.json path")
    p.add_argument("--layers", type=int, default=40)
    p.add_argument("--seq-len", type=int, default=4096)
    p.add_argument("--batch-size", type=int, default=1)
    p.add_argument("--lora-rank", type=int, default=16)
    p.add_argument("--learning-rate", type=float, default=1e-4)
    p.add_argument("--no-gradient-checkpointing", action="store_true")
    p.add_argument("--device", default="auto", help="auto, cuda or cpu")
    return p.parse_args(argv)


def expert_bytes_per_rank(cfg, world: int) -> float:
    """Packed MXFP4 routed experts of this rank: 0.5 byte per value + one scale byte per 32."""
    per_expert = 3 * cfg.hidden_size * cfg.moe_intermediate_size * (0.5 + 1 / 32)
    return cfg.num_hidden_layers * (cfg.n_routed_experts / world) * per_expert


def emit(record: dict) -> None:
    print(json.dumps(record), flush=True)


def main(argv=None) -> None:
    args = parse_args(argv)
    import torch
    import torch.distributed as dist

    from tiny_dsv41_b200.lora import LoRAConfig, adapter_parameters, inject_lora
    from tiny_dsv41_b200.models.dsv4 import DeepSeekV41Config
    from tiny_dsv41_b200.models.dsv4.checkpoint import prefix_config
    from tiny_dsv41_b200.models.dsv4.synthetic import build_synthetic_backbone

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    use_cuda = args.device == "cuda" or (args.device == "auto" and torch.cuda.is_available())
    device = torch.device("cuda", local) if use_cuda else torch.device("cpu")
    if use_cuda:
        torch.cuda.set_device(device)
    cfg = prefix_config(DeepSeekV41Config.from_json(CONFIGS.get(args.config, args.config)), args.layers)
    base = {"metric": METRIC, "impl": "native", "n_gpus": world if use_cuda else 0, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
            "dtype": "bf16" if use_cuda else "fp32", "data": "synthetic", "unit": "tokens/s",
            "config": {"model": f"DeepSeek-V4.1-{args.config} {args.layers}-layer prefix, LoRA r{args.lora_rank} "
                                f"on q_a/q_b, frozen MXFP4 experts, Engram offload, mHC",
                       "global_batch": args.batch_size * world, "seq_len": args.seq_len,
                       "parallelism": f"ep{world}"}}
    need = expert_bytes_per_rank(cfg, world)
    if use_cuda and need > HBM_BYTES - ACTIVATION_RESERVE:
        if rank == 0:
            emit({**base, "value": None, "unavailable": f"the packed experts need {need / 2 ** 30:.0f} GiB per rank "
                                                        f"at EP{world}; run with 8 GPUs"})
        return
    if world > 1:
        dist.init_process_group("nccl" if use_cuda else "gloo", timeout=timedelta(minutes=10))
    meshes, dispatcher = None, None
    if world > 1:
        from tiny_dsv41_b200.parallel.meshes import ParallelMeshes

        meshes = ParallelMeshes.build(cp=1, ep=world, device_type=device.type, engram=True)
        if use_cuda:
            from tiny_dsv41_b200.parallel.nvlink_ep import NVLinkTokenDispatcher

            dispatcher = NVLinkTokenDispatcher(meshes.ep, max_tokens=args.batch_size * args.seq_len)
        else:
            from tiny_dsv41_b200.parallel.dispatch import AllToAllTokenDispatcher

            dispatcher = AllToAllTokenDispatcher(meshes.ep)
    dtype = torch.bfloat16 if use_cuda else torch.float32
    began = time.monotonic()
    model = build_synthetic_backbone(cfg, device=device, dtype=dtype, token_dispatcher=dispatcher,
                                     engram_mesh=meshes.engram if meshes is not None else None,
                                     sparse_engram_gradients=True, engram_offload=True, fp4_experts=True,
                                     seed=1234 + rank)
    build_seconds = time.monotonic() - began
    for layer in model.model.layers:
        if layer.attention.indexer is not None:
            layer.attention.indexer.stable_topk = True
    inject_lora(model, LoRAConfig(args.lora_rank, 2.0 * args.lora_rank, 0.0, ("attention.q_a", "attention.q_b")))
    adapters = list(adapter_parameters(model))
    keep = {id(p) for p in adapters}
    for p in model.parameters():
        if id(p) not in keep:
            p.requires_grad_(False)
    if not args.no_gradient_checkpointing:
        model.gradient_checkpointing_enable()
    model.train()
    optimizer = torch.optim.AdamW(adapters, lr=args.learning_rate, fused=use_cuda)
    generator = torch.Generator(device=device).manual_seed(7 + rank)

    def step() -> torch.Tensor:
        ids = torch.randint(0, cfg.vocab_size, (args.batch_size, args.seq_len), device=device, generator=generator)
        loss = model(ids, labels=ids).loss
        loss.backward()
        if world > 1:  # adapters are data-parallel over all ranks: one flat averaged all-reduce
            grads = [p.grad for p in adapters]
            flat = torch.cat([g.reshape(-1) for g in grads])
            dist.all_reduce(flat)
            flat.div_(world)
            offset = 0
            for g in grads:
                g.copy_(flat[offset:offset + g.numel()].view_as(g))
                offset += g.numel()
        optimizer.step()
        optimizer.zero_grad(set_to_none=True)
        return loss.detach()

    def sync() -> None:
        if world > 1:
            dist.barrier()
        if use_cuda:
            torch.cuda.synchronize()

    for _ in range(args.warmup):
        step()
    sync()
    clocks = None
    if use_cuda:
        from bench import ClockSampler

        sampler = ClockSampler(device.index)
        sampler.__enter__()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
    else:
        t0 = time.perf_counter()
    for _ in range(args.steps):
        loss = step()
    if use_cuda:
        end.record()
        torch.cuda.synchronize()
        ms = start.elapsed_time(end) / args.steps
        sampler.__exit__(None, None, None)
        clocks = sampler.summary()
    else:
        ms = (time.perf_counter() - t0) * 1000 / args.steps
    sync()
    if world > 1:
        worst = torch.tensor([ms], dtype=torch.float64, device=device if use_cuda else "cpu")
        dist.all_reduce(worst, op=dist.ReduceOp.MAX)
        ms = float(worst.item())
    tokens = args.batch_size * args.seq_len * world
    if rank == 0:
        record = {**base, "value": tokens * 1000.0 / ms, "ms_per_step": ms, "vs_baseline": None,
                  "loss": float(loss.item()), "build_seconds": round(build_seconds, 1),
                  "expert_gib_per_rank": round(need / 2 ** 30, 1),
                  "adapter_parameters": sum(p.numel() for p in adapters)}
        if clocks is not None:
            record["clocks"] = clocks
        emit(record)
    if world > 1:
        if dispatcher is not None and hasattr(dispatcher, "close"):
            dispatcher.close()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
