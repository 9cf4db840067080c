"""Text SFT (full or LoRA) for DeepSeek-V4.1 and Qwen3-MoE checkpoints: the ``train_sft.py`` CLI.

Flow and flags of the reference driver (``train_sft.py:26-452``): validate arguments -> run
identity (config / base files / data hashes + training config) -> load the base model with this
rank's experts and (optionally) LoRA adapters -> FSDP2 -> optimizer (AdamW or SGD; LoRA defaults
to AdamW, full to SGD) -> optional resume from a same-topology snapshot -> baseline evaluation
-> ``--steps`` optimizer steps of ``--gradient-accumulation-steps`` micro-batches -> snapshots
every ``--save-every`` steps and at the end -> final evaluation -> LoRA adapter export ->
``summary.json``. Metrics stream as JSON lines to stdout and ``metrics.jsonl``.

Gradients are normalised by the global number of supervised tokens of the whole step (every
micro-batch of every data-parallel rank), not per batch. Data: each data-parallel group reads a
deterministic cyclic window of the examples (``make_batches``); context-parallel ranks of one
group read the same batch and split its sequence.

Launch with torchrun (one process per GPU); a single process also runs (CPU or one GPU).
"""

from __future__ import annotations

import argparse
import json
import math
import time
from dataclasses import asdict
from pathlib import Path

import torch
import torch.distributed as dist

from ..ops import StatusMonitor
from ..lora import LoRAConfig, adapter_parameters, inject_lora, save_adapter
from ..parallel.fsdp import scale_expert_grads
from ..rl.checkpoint import run_identity
from ..rl.tokenizer import ModelTokenizer
from ..runtime import initialize_runtime, local_tensor
from ..utils.trace import trace_point
from .sft_checkpoint import load_checkpoint, save_checkpoint
from .sft_data import collate_examples, load_jsonl

QWEN_LORA_TARGETS = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj")


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--model-path", required=True)
    p.add_argument("--data", required=True, help="JSONL prompt/answer or messages/answer records")
    p.add_argument("--eval-data", help="defaults to the training data")
    p.add_argument("--output-dir", required=True)
    p.add_argument("--family", choices=("dsv4", "qwen"), default="dsv4")
    p.add_argument("--mode", choices=("full", "lora"), default="lora")
    p.add_argument("--num-layers", type=int, help="DSV4 backbone prefix; default is the whole backbone")
    p.add_argument("--steps", type=int, default=20, help="total optimizer steps (0 = evaluate only)")
    p.add_argument("--batch-size", type=int, default=1)
    p.add_argument("--gradient-accumulation-steps", type=int, default=1)
    p.add_argument("--seq-len", type=int, default=4096, help="token limit per example (no truncation)")
    p.add_argument("--learning-rate", type=float, default=1e-4)
    p.add_argument("--optimizer", choices=("sgd", "adamw"))
    p.add_argument("--cp-size", type=int, default=1)
    p.add_argument("--ep-size", type=int, default=1)
    p.add_argument("--lora-rank", type=int, default=8)
    p.add_argument("--lora-alpha", type=float, default=16.0)
    p.add_argument("--lora-dropout", type=float, default=0.0)
    p.add_argument("--lora-targets", help="comma-separated layer-relative linear module suffixes")
    p.add_argument("--engram-offload", action="store_true", help="keep DSV4 Engram rows in host memory")
    p.add_argument("--train-engram", action="store_true", help="also update Engram tables in LoRA mode (SGD)")
    p.add_argument("--fp4-experts", action="store_true",
                   help="DSV4 LoRA: keep the frozen routed experts as MXFP4 codes, multiplied packed")
    p.add_argument("--gradient-checkpointing", action="store_true")
    p.add_argument("--seed", type=int, default=42)
    p.add_argument("--eval-batches", type=int, default=1, help="fixed evaluation batches per data group")
    p.add_argument("--generation-eval", action="store_true", help="also greedy-decode the evaluation prompts")
    p.add_argument("--generation-max-new-tokens", type=int, default=16)
    p.add_argument("--save-every", type=int, default=0)
    p.add_argument("--no-save", action="store_true", help="skip snapshots and adapter export")
    p.add_argument("--resume", help="same-topology SFT snapshot directory")
    p.add_argument("--device", default="auto", help="auto, cuda or cpu")
    return p.parse_args(argv)


def validate_args(args, world_size: int) -> None:
    if args.steps < 0 or args.save_every < 0:
        raise ValueError("steps and save-every must be nonnegative")
    if args.no_save and args.save_every:
        raise ValueError("no-save cannot be combined with save-every")
    if min(args.batch_size, args.gradient_accumulation_steps, args.eval_batches,
           args.generation_max_new_tokens) < 1 or args.seq_len < 2:
        raise ValueError("batch-size, accumulation and eval-batches must be positive; seq-len at least 2")
    if not math.isfinite(args.learning_rate) or args.learning_rate <= 0:
        raise ValueError("learning-rate must be positive and finite")
    if min(args.cp_size, args.ep_size) < 1 or world_size % args.cp_size or world_size % args.ep_size:
        raise ValueError("cp-size and ep-size must divide world size")
    if args.family != "dsv4" and (args.engram_offload or args.train_engram):
        raise ValueError("Engram options require the DSV4 model family")
    if args.fp4_experts and (args.family != "dsv4" or args.mode != "lora"):
        raise ValueError("fp4-experts keeps experts frozen: it requires DSV4 LoRA")
    if args.seq_len % args.cp_size:
        raise ValueError("seq-len must divide evenly across cp-size")
    for name in ("config.json", "model.safetensors.index.json"):
        if not (Path(args.model_path) / name).is_file():
            raise FileNotFoundError(Path(args.model_path) / name)
    if args.family == "dsv4":
        from ..models.dsv4 import DeepSeekV41Config

        config = DeepSeekV41Config.from_json(Path(args.model_path) / "config.json")
        args.num_layers = config.num_hidden_layers if args.num_layers is None else args.num_layers
        if not 1 <= args.num_layers <= config.num_hidden_layers:
            raise ValueError("num-layers must select a nonempty DSV4 backbone prefix")
        experts = config.n_routed_experts
    else:
        from ..models.qwen import Qwen3MoeConfig

        if args.num_layers is not None:
            raise ValueError("num-layers is supported only for DSV4")
        experts = Qwen3MoeConfig.from_json(Path(args.model_path) / "config.json").num_experts
    if experts % args.ep_size:
        raise ValueError("expert count must divide evenly across ep-size")
    args.optimizer = args.optimizer or ("sgd" if args.mode == "full" or args.train_engram else "adamw")
    if (args.train_engram or (args.engram_offload and args.mode == "full")) and args.optimizer != "sgd":
        raise ValueError("trainable offloaded Engram requires SGD")


def _backbone_layers(args) -> int:
    from ..models.dsv4 import DeepSeekV41Config

    return DeepSeekV41Config.from_json(Path(args.model_path) / "config.json").num_hidden_layers


def lora_config(args) -> LoRAConfig:
    defaults = LoRAConfig().targets if args.family == "dsv4" else QWEN_LORA_TARGETS
    targets = tuple(n.strip() for n in args.lora_targets.split(",")) if args.lora_targets else defaults
    return LoRAConfig(args.lora_rank, args.lora_alpha, args.lora_dropout, targets)


def load_model(args, runtime):
    """Base weights for this rank, LoRA adapters, then FSDP2 (multi-process runs)."""
    from ..parallel.cp import ContextParallel
    from ..parallel.dispatch import TokenDispatcher

    distributed = dist.is_initialized() and dist.get_world_size() > 1
    meshes, cp, dispatcher = None, ContextParallel(), TokenDispatcher()
    if distributed:
        from ..parallel.meshes import ParallelMeshes

        meshes = ParallelMeshes.build(cp=args.cp_size, ep=args.ep_size, device_type=runtime.device.type,
                                      engram=args.family == "dsv4")
        cp = ContextParallel(meshes.cp)
        if meshes.ep is not None:
            if runtime.device.type == "cuda":
                from ..parallel.nvlink_ep import NVLinkTokenDispatcher

                dispatcher = NVLinkTokenDispatcher(meshes.ep, max_tokens=args.batch_size * args.seq_len)
            else:
                from ..parallel.dispatch import AllToAllTokenDispatcher

                dispatcher = AllToAllTokenDispatcher(meshes.ep)
    dtype = torch.bfloat16 if runtime.device.type == "cuda" else torch.float32
    if args.family == "dsv4":
        from ..models.dsv4.checkpoint import load_dsv41_backbone_window

        model = load_dsv41_backbone_window(
            args.model_path, num_layers=args.num_layers, device=runtime.device, dtype=dtype, context_parallel=cp,
            token_dispatcher=dispatcher, engram_mesh=meshes.engram if meshes is not None else None,
            sparse_engram_gradients=args.mode == "lora" or args.optimizer == "sgd",
            engram_offload=args.engram_offload, fp4_experts=args.fp4_experts)
        for layer in model.model.layers:
            if layer.attention.indexer is not None:
                layer.attention.indexer.stable_topk = True
    else:
        from ..models.qwen import load_qwen3_moe

        model = load_qwen3_moe(args.model_path, device=runtime.device, dtype=dtype, context_parallel=cp,
                               token_dispatcher=dispatcher)
    if args.mode == "lora":
        inject_lora(model, lora_config(args))
        keep = {id(p) for p in adapter_parameters(model)}
        for p in model.parameters():
            if id(p) not in keep:
                p.requires_grad_(False)
        if args.family == "dsv4":
            model.model.engram_tables.requires_grad_(args.train_engram)
    if args.gradient_checkpointing:
        model.gradient_checkpointing_enable()
    if distributed:
        from ..parallel.fsdp import apply_fsdp

        apply_fsdp(model, meshes, param_dtype=dtype)
    return model, meshes


def make_batches(examples, cursor: int, *, batch_size: int, count: int, runtime, cp_size: int, pad_token_id: int):
    """Identical data within a CP group; a deterministic global cyclic cursor."""
    data_size, data_rank = runtime.world_size // cp_size, runtime.rank // cp_size
    batches = []
    for micro in range(count):
        start = cursor + (micro * data_size + data_rank) * batch_size
        selected = [examples[(start + i) % len(examples)] for i in range(batch_size)]
        batches.append(collate_examples(selected, pad_token_id=pad_token_id, pad_to_multiple_of=cp_size))
    return batches, cursor + count * data_size * batch_size


def _step_resources(model, runtime, seconds: float) -> dict:
    """Step seconds and peak device memory (max over ranks) and the Engram row-cache counters (sum
    over ranks) of the offloaded tables; the reference's SFT step record (``train_sft.py:347-436``)."""
    peak = [seconds, 0.0, 0.0]
    if runtime.device.type == "cuda":
        peak[1] = torch.cuda.max_memory_allocated(runtime.device) / 2 ** 30
        peak[2] = torch.cuda.max_memory_reserved(runtime.device) / 2 ** 30
    peak_t = _reduce(torch.tensor(peak, device=runtime.device, dtype=torch.float64), runtime,
                     dist.ReduceOp.MAX if dist.is_initialized() else None)
    out = {"seconds": peak_t[0].item()}
    if runtime.device.type == "cuda":
        out.update(peak_allocated_gib=round(peak_t[1].item(), 3), peak_reserved_gib=round(peak_t[2].item(), 3))
    lookups = [m._cpu_lookup for m in model.modules() if getattr(m, "_cpu_lookup", None) is not None]
    if lookups:
        keys = ("hits", "misses", "transferred_rows")
        counts = torch.tensor([sum(lk.cache_metrics[k] for lk in lookups) for k in keys], device=runtime.device,
                              dtype=torch.float64)
        counts = _reduce(counts, runtime)
        out.update({f"engram_cache_{k}": int(v) for k, v in zip(keys, counts.tolist())})
    return out


def _reduce(value, runtime, op=None):
    if dist.is_initialized():
        dist.all_reduce(value, op=op or dist.ReduceOp.SUM)
    return value


def _loss(model, batch, family, runtime):
    options = {"compute_aux_loss": False} if family == "dsv4" else {"output_router_logits": False}
    loss = model(**{k: v.to(runtime.device) for k, v in batch.items()}, **options).loss
    finite = torch.isfinite(loss.detach()).to(torch.int32)
    if not _reduce(finite, runtime, dist.ReduceOp.MIN if dist.is_initialized() else None).item():
        raise RuntimeError("SFT produced a non-finite loss")
    return loss


def train_update(model, optimizer, batches, *, family, runtime, cp_size=1, ep_size=1) -> dict:
    counts = [int((b["labels"][:, 1:] != -100).sum()) for b in batches]
    totals = torch.tensor([sum(counts), sum(int(b["attention_mask"].sum()) for b in batches)],
                          device=runtime.device, dtype=torch.float64)
    totals = _reduce(totals, runtime) / cp_size
    if not counts or min(counts) == 0 or totals[0].item() <= 0:
        raise ValueError("each SFT micro-batch must contain supervised next-token targets")
    optimizer.zero_grad(set_to_none=True)
    weighted = torch.zeros((), device=runtime.device, dtype=torch.float64)
    model.train()
    for batch, count in zip(batches, counts):
        loss = _loss(model, batch, family, runtime)
        (loss * ((runtime.world_size // cp_size) * count / totals[0])).backward()
        weighted += loss.detach().double() * count
    scale_expert_grads(model, ep_size)
    finite = torch.ones((), device=runtime.device, dtype=torch.int32)
    for p in model.parameters():
        if p.requires_grad and p.grad is not None:
            g = local_tensor(p.grad)
            if g.is_sparse:
                g = g.coalesce().values()
            finite &= torch.isfinite(g).all().to(device=runtime.device, dtype=torch.int32)
    if not _reduce(finite, runtime, dist.ReduceOp.MIN if dist.is_initialized() else None).item():
        raise RuntimeError("SFT produced a non-finite gradient; reload the last snapshot")
    optimizer.step()
    loss_value = (_reduce(weighted, runtime) / cp_size / totals[0]).item()
    return {"loss": loss_value, "supervised_tokens": int(totals[0].item()), "input_tokens": int(totals[1].item())}


@torch.no_grad()
def evaluate(model, batches, *, family, runtime, cp_size=1) -> float:
    was = model.training
    model.eval()
    totals = torch.zeros(2, device=runtime.device, dtype=torch.float64)
    try:
        for batch in batches:
            count = int((batch["labels"][:, 1:] != -100).sum())
            totals[0] += _loss(model, batch, family, runtime).double() * count
            totals[1] += count
        totals = _reduce(totals, runtime) / cp_size
        if totals[1].item() <= 0:
            raise ValueError("evaluation requires supervised tokens")
        return (totals[0] / totals[1]).item()
    finally:
        model.train(was)


def _identity(args, runtime) -> dict:
    identity = run_identity(args.model_path, args.data, False, eval_data_path=args.eval_data)
    identity["training_config"] = {k: getattr(args, k) for k in (
        "family", "mode", "num_layers", "batch_size", "gradient_accumulation_steps", "seq_len", "learning_rate",
        "optimizer", "cp_size", "ep_size", "seed", "gradient_checkpointing")}
    identity["training_config"].update({k: True for k in ("engram_offload", "train_engram") if getattr(args, k)})
    identity["training_config"].update(world_size=runtime.world_size, enable_thinking=False,
                                       lora=asdict(lora_config(args)) if args.mode == "lora" else None)
    return json.loads(json.dumps(identity))


def train(args, runtime) -> dict:
    validate_args(args, runtime.world_size)
    torch.manual_seed(args.seed)
    tokenizer = ModelTokenizer(args.model_path)
    examples = load_jsonl(args.data, tokenizer, max_length=args.seq_len)
    eval_examples = load_jsonl(args.eval_data, tokenizer, max_length=args.seq_len) if args.eval_data else examples
    identity = _identity(args, runtime)
    started = time.perf_counter()
    model, _ = load_model(args, runtime)
    load_seconds = time.perf_counter() - started
    params = [p for p in model.parameters() if p.requires_grad]
    opt_type = torch.optim.SGD if args.optimizer == "sgd" else torch.optim.AdamW
    optimizer = opt_type(params, lr=args.learning_rate, weight_decay=0, foreach=False)
    if args.family == "dsv4" and args.optimizer == "sgd" and (args.mode == "full" or args.train_engram):
        from ..parallel.engram_offload import install_engram_sgd_hooks
        from .sft_engram import build_engram_checkpoint

        install_engram_sgd_hooks(model, optimizer)
        model._sft_engram_checkpoint = build_engram_checkpoint(model, args.model_path, optimizer)
    step, cursor = load_checkpoint(args.resume, model, optimizer, identity=identity) if args.resume else (0, 0)
    expected = step * args.gradient_accumulation_steps * args.batch_size * (runtime.world_size // args.cp_size)
    if cursor != expected:
        raise ValueError("checkpoint data cursor does not match completed SFT steps")
    if args.steps and step > args.steps:
        raise ValueError("resume step exceeds the requested total steps")
    initial = step
    out = Path(args.output_dir)
    if runtime.is_main:
        out.mkdir(parents=True, exist_ok=True)

    def emit(event):
        if runtime.is_main:
            print(json.dumps(event), flush=True)
            with (out / "metrics.jsonl").open("a", encoding="utf-8") as f:
                f.write(json.dumps(event) + "\n")

    options = dict(batch_size=args.batch_size, runtime=runtime, cp_size=args.cp_size,
                   pad_token_id=tokenizer.eos_token_ids[0])
    eval_batches, _ = make_batches(eval_examples, 0, count=args.eval_batches, **options)

    def generation_eval():
        if not args.generation_eval:
            return None
        from .sft_eval import evaluate_answers

        count = args.eval_batches * args.batch_size * (runtime.world_size // args.cp_size)
        return evaluate_answers(model, eval_examples[:count], tokenizer, max_new_tokens=args.generation_max_new_tokens,
                                device=runtime.device)

    before = evaluate(model, eval_batches, family=args.family, runtime=runtime, cp_size=args.cp_size)
    gen_before = generation_eval()
    emit({"event": "loaded", "step": step, "eval_loss_before": before, "generation_before": gen_before,
          "load_seconds": load_seconds})
    saved = None
    monitor = StatusMonitor(runtime.device)
    loop_started = time.perf_counter()
    for step in range(initial + 1, args.steps + 1):
        batches, next_cursor = make_batches(examples, cursor, count=args.gradient_accumulation_steps, **options)
        trace_point("step_begin", step=step, data_position=cursor)
        t0 = time.perf_counter()
        metrics = train_update(model, optimizer, batches, family=args.family, runtime=runtime, cp_size=args.cp_size,
                               ep_size=args.ep_size)
        if runtime.device.type == "cuda":
            torch.cuda.synchronize(runtime.device)
        monitor.step_end(f"SFT step {step}")
        metrics.update(_step_resources(model, runtime, time.perf_counter() - t0))
        trace_point("step_end", step=step, seconds=metrics["seconds"])
        cursor = next_cursor
        emit({"event": "train", "step": step, "data_position": cursor, **metrics})
        if not args.no_save and args.save_every and step % args.save_every == 0:
            save_checkpoint(out / f"checkpoint-{step:08d}", model, optimizer, step=step, identity=identity,
                            data_position=cursor)
            saved = step
    loop_seconds = time.perf_counter() - loop_started
    if not args.no_save and step > initial and step != saved:
        save_checkpoint(out / f"checkpoint-{step:08d}", model, optimizer, step=step, identity=identity,
                        data_position=cursor)
    optimizer.zero_grad(set_to_none=True)
    after = evaluate(model, eval_batches, family=args.family, runtime=runtime, cp_size=args.cp_size)
    gen_after = generation_eval()
    if not args.no_save and args.mode == "lora" and step > 0 and (step > initial or args.resume):
        if args.train_engram:
            if args.engram_offload and args.lora_dropout == 0 and args.num_layers == _backbone_layers(args):
                from .sft_export import export_sft_bundle

                snapshot = Path(args.resume) if step == initial else out / f"checkpoint-{step:08d}"
                bundle = export_sft_bundle(model, snapshot, args.model_path, out / f"sft-bundle-{step:08d}")
                emit({"event": "sft_bundle_exported", "step": step, "path": str(bundle)})
            else:
                emit({"event": "sft_bundle_unavailable",
                      "reason": "requires the complete backbone, dropout=0 and host-memory Engram"})
        else:
            base = {k: v for k, v in identity.items() if k not in {"training_config", "data_sha256", "eval_data_sha256"}}
            save_adapter(model, out / "adapter.pt", base_identity=base)
            if runtime.is_main:
                (out / "adapter_metadata.json").write_text(json.dumps({"identity": identity, "step": step}, indent=2) + "\n")
    summary = {"event": "summary", "step": step, "initial_step": initial, "data_position": cursor,
               "checkpoint_saving": not args.no_save, "eval_loss_before": before, "eval_loss_after": after,
               "load_seconds": load_seconds, "loop_seconds": loop_seconds, "generation_before": gen_before,
               "generation_after": gen_after}
    emit(summary)
    if runtime.is_main:
        (out / "summary.json").write_text(json.dumps(summary, indent=2) + "\n", encoding="utf-8")
    return summary


def main(argv=None) -> None:
    runtime = None
    try:
        args = parse_args(argv)
        runtime = initialize_runtime(args.device, require_distributed=True)
        train(args, runtime)
    finally:
        if runtime is not None and dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
