"""``train.py``: train the tiny DeepSeek-V4.1 causal LM on synthetic, learnable sequences.

Behaviour of the reference's ``train.py``: every rank builds identical random-init weights
(seeded), FSDP2 shards them in multi-process runs, each rank draws its own batches of
``bos, s, s+1, ...`` (mod vocab) sequences from a per-rank generator, AdamW with global-norm
clipping at 1.0, JSON progress lines, and a DCP checkpoint at the end.
"""

from __future__ import annotations

import argparse
import json
from pathlib import Path

import torch
import torch.distributed as dist

from ..checkpoint import CheckpointManager, TrainingState
from ..models.dsv4 import DeepSeekV41Config, DeepSeekV41ForCausalLM
from ..runtime import distributed_mean, initialize_runtime

ROOT = Path(__file__).resolve().parents[2]


def parse_args(argv=None):
    p = argparse.ArgumentParser(description="Train a tiny DeepSeek V4.1 causal LM")
    p.add_argument("--model-config", default=str(ROOT / "tiny_dsv41_b200/models/dsv4/tiny_config.json"))
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--batch-size", type=int, default=4)
    p.add_argument("--seq-len", type=int, default=32)
    p.add_argument("--learning-rate", type=float, default=3e-4)
    p.add_argument("--device", default="auto")
    p.add_argument("--log-every", type=int, default=1)
    p.add_argument("--output-dir", default="outputs/final")
    p.add_argument("--seed", type=int, default=42)
    p.add_argument("--resume", action="store_true", help="continue from the latest checkpoint in output-dir")
    p.add_argument("--local-rank", "--local_rank", type=int, default=None, help=argparse.SUPPRESS)
    return p.parse_args(argv)


def make_batch(batch_size, seq_len, device, *, config, generator=None) -> torch.Tensor:
    starts = torch.randint(config.vocab_size, (batch_size, 1), device=device, generator=generator)
    body = (starts + torch.arange(seq_len - 1, device=device).unsqueeze(0)) % config.vocab_size
    bos = torch.full((batch_size, 1), config.bos_token_id, dtype=torch.long, device=device)
    return torch.cat((bos, body), dim=1)


def clip_grad_norm(parameters, max_norm: float) -> torch.Tensor:
    norm = torch.nn.utils.clip_grad_norm_(list(parameters), max_norm, foreach=False)
    if hasattr(norm, "full_tensor"):
        norm = norm.full_tensor()
    return norm.detach().float()


def validate_args(args) -> None:
    if args.steps < 1 or args.batch_size < 1 or args.log_every < 1:
        raise ValueError("steps, batch-size, and log-every must be positive")
    config = DeepSeekV41Config.from_json(args.model_config)
    if not 2 <= args.seq_len <= config.max_position_embeddings:
        raise ValueError("seq-len must be between 2 and the configured max_position_embeddings")


def train(args, runtime) -> dict:
    torch.manual_seed(args.seed)
    config = DeepSeekV41Config.from_json(args.model_config)
    model = DeepSeekV41ForCausalLM(config)
    count = sum(p.numel() for p in model.parameters())
    model = model.to(runtime.device)
    if runtime.device.type == "cuda":
        model.to_mixed_precision(torch.bfloat16)
    if runtime.distributed:
        from ..parallel.fsdp import apply_fsdp
        from ..parallel.meshes import ParallelMeshes

        apply_fsdp(model, ParallelMeshes.build(device_type=runtime.device.type),
                   param_dtype=torch.bfloat16 if runtime.device.type == "cuda" else torch.float32)
    optimizer = torch.optim.AdamW(model.parameters(), lr=args.learning_rate)
    generator = torch.Generator(device=runtime.device)
    generator.manual_seed(args.seed + runtime.rank)
    manager = CheckpointManager(Path(args.output_dir) / "checkpoint",
                                TrainingState(model, optimizer, model_config=config.to_dict(), data_generator=generator))
    start = manager.load() if args.resume and manager.latest_step() is not None else 0
    if runtime.is_main:
        print(json.dumps({"device": str(runtime.device), "world_size": runtime.world_size,
                          "parallelism": "fsdp" if runtime.distributed else "none", "parameters": count,
                          "global_batch_size": args.batch_size * runtime.world_size, "start_step": start}), flush=True)
    loss_value = None
    for step in range(start + 1, args.steps + 1):
        ids = make_batch(args.batch_size, args.seq_len, runtime.device, config=config, generator=generator)
        optimizer.zero_grad(set_to_none=True)
        loss = model(input_ids=ids, attention_mask=torch.ones_like(ids), labels=ids).loss
        loss.backward()
        norm = clip_grad_norm(model.parameters(), 1.0)
        optimizer.step()
        if step % args.log_every == 0 or step == args.steps:
            loss_value = distributed_mean(loss, runtime)
            if runtime.is_main:
                print(json.dumps({"step": step, "loss": loss_value, "grad_norm": norm.item()}), flush=True)
    path = manager.save(args.steps)
    if runtime.is_main:
        print(f"saved checkpoint to {path}", flush=True)
    return {"loss": loss_value, "checkpoint": str(path)}


def main(argv=None) -> None:
    args = parse_args(argv)
    validate_args(args)
    runtime = None
    try:
        runtime = initialize_runtime(args.device, args.local_rank)
        train(args, runtime)
    finally:
        if runtime is not None and runtime.distributed and dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
