"""Reference arm of ``bench.py``: the unmodified reference package (installed under
``baseline/_ref``) driven through its own public API on the same metric and config.

Stock path, as in the reference's ``train_qwen.py``: ``Qwen3MoeForCausalLM`` with
``AllToAllTokenDispatcher`` (EP = N), ``apply_fsdp2`` (FSDP2 over the world, bf16 parameters,
fp32 reduction), ``ParallelParameters`` gradient clipping and ``torch.optim.AdamW``. The
reference drivers require cp == ep, so the meshes are built directly with
``ParallelMeshes.build(cp=1, ep=N)`` as the benchmark config asks. Only the harness (synthetic
tokens, on-device random init with std 0.02, timing) is ours.
"""

from __future__ import annotations

import os
import time


def _unavailable(args, metric, model, why):
    return {"metric": metric, "impl": "reference", "unavailable": why, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "value": None,
            "config": {"model": model, "seq_len": args.seq_len}}


def run_reference_arm(args, metric: str, model_name: str):
    try:
        import dsv41_train  # noqa: F401
        from dsv41_train.cp import ContextParallel
        from dsv41_train.dispatch import AllToAllTokenDispatcher, TokenDispatcher
        from dsv41_train.models.qwen.config import Qwen3MoeConfig
        from dsv41_train.models.qwen.model import Qwen3MoeForCausalLM
        from dsv41_train.models.qwen.parallel import ParallelParameters, apply_fsdp2
        from dsv41_train.parallel import ParallelMeshes
        from dsv41_train.runtime import initialize_runtime
    except Exception as error:  # pragma: no cover - depends on the install
        return _unavailable(args, metric, model_name, f"reference not importable from baseline/_ref: {error!r}")
    import torch
    import torch.distributed as dist

    if args.layers != 48:
        model_name = f"REDUCED {args.layers}L (not the benchmark)"
    # A one-GPU run is started without torchrun: give the reference's runtime the single-rank
    # environment it reads, and open the process group here with a bounded timeout so a rank that
    # fails (for instance out of memory) ends its peers' next collective with an error, not a hang.
    for key, value in (("RANK", "0"), ("LOCAL_RANK", "0"), ("WORLD_SIZE", "1"), ("MASTER_ADDR", "127.0.0.1"),
                       ("MASTER_PORT", "29533")):
        os.environ.setdefault(key, value)
    if not dist.is_initialized():
        import datetime

        torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
        dist.init_process_group(backend="nccl", timeout=datetime.timedelta(seconds=300))
    runtime = initialize_runtime(require_distributed=True)
    world = runtime.world_size
    try:
        cp_size = getattr(args, "cp", 1)
        meshes = ParallelMeshes.build(cp=cp_size, ep=world, device_type="cuda")
        dispatcher = AllToAllTokenDispatcher(meshes.ep) if meshes.ep is not None else TokenDispatcher()
        config = Qwen3MoeConfig(num_hidden_layers=args.layers, max_window_layers=args.layers)
        cp = ContextParallel(meshes.cp)
        with torch.device("meta"):
            model = Qwen3MoeForCausalLM(config, cp, dispatcher)
        # bf16 storage from the start, as the stock loader (load_qwen3_moe with dtype=bf16) assigns it
        model = model.to(torch.bfloat16).to_empty(device=runtime.device)
        gen = torch.Generator(device="cuda")
        gen.manual_seed(1 + runtime.rank)
        with torch.no_grad():
            for name, p in model.named_parameters():
                if name.endswith("norm.weight") or "layernorm" in name:
                    p.fill_(1.0)
                else:
                    p.normal_(0.0, config.initializer_range, generator=gen)
        model.gradient_checkpointing_enable()
        model.train()
        apply_fsdp2(model, meshes)
        parameters = ParallelParameters.collect(model)
        optimizer = torch.optim.AdamW(model.parameters(), lr=args.lr, foreach=False)

        # the ranks of one CP group train on the same sequences (the model keeps each rank's chunk)
        host = torch.Generator().manual_seed(1234 + runtime.rank // cp_size)
        batches = []
        for _ in range(4):
            ids = torch.randint(0, config.vocab_size, (args.batch_size, args.seq_len), generator=host)
            ids[:, 0] = config.bos_token_id
            labels = ids.clone()
            labels[:, : args.seq_len // 2] = -100
            batches.append((ids.pin_memory(), labels.pin_memory()))

        def step(i):
            ids, labels = batches[i % len(batches)]
            ids = ids.to(runtime.device, non_blocking=True)
            labels = labels.to(runtime.device, non_blocking=True)
            optimizer.zero_grad(set_to_none=True)
            out = model(ids, labels=labels, output_router_logits=True)
            out.loss.backward()
            parameters.synchronize(cp)
            parameters.clip_grad_norm(cp)
            optimizer.step()
            return out.loss.detach()

        for i in range(args.warmup):
            step(i)
        flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=runtime.device)
        dist.barrier()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for i in range(args.steps):
            flush.zero_()
            step(i)
        end.record()
        dist.barrier()
        torch.cuda.synchronize()
        device_ms = start.elapsed_time(end)
        wall0 = time.perf_counter()
        for i in range(args.steps):
            step(i).item()
        torch.cuda.synchronize()
        wall_ms = (time.perf_counter() - wall0) * 1000
        times = torch.tensor([device_ms, wall_ms], device=runtime.device)
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
        device_ms, wall_ms = times.tolist()
        tokens = args.batch_size * args.seq_len * (world // cp_size) * args.steps
        record = {
            "metric": metric, "impl": "reference", "value": tokens / (device_ms / 1000), "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": device_ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "dtype": "bf16", "data": "synthetic", "vs_baseline": None,
            "e2e": {"value": tokens / (wall_ms / 1000), "unit": "tokens/s",
                    "h2d_bytes_per_step": 2 * args.batch_size * args.seq_len * 8, "d2h_bytes_per_step": 4},
            "config": {"model": model_name, "global_batch": args.batch_size * world // cp_size,
                       "seq_len": args.seq_len,
                       "parallelism": (f"cp{cp_size}+" if cp_size > 1 else "") + f"ep{world}+fsdp{world // cp_size}",
                       "optimizer": "torch AdamW on bf16 params (stock)",
                       "grad_ckpt": True, "l2": "256 MB buffer written between timed steps"},
        }
    except torch.OutOfMemoryError as error:
        record = _unavailable(args, metric, model_name, f"reference ran out of GPU memory at N={world}: "
                              f"{str(error).splitlines()[0][:200]}")
    finally:
        if dist.is_initialized():
            try:
                dist.barrier()
            except Exception:
                pass
            dist.destroy_process_group()
    return record
