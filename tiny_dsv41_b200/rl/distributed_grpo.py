"""Distributed query-LoRA GRPO against a persistent rollout service
(``dsv41_train/rl/distributed_grpo.py:37-641``, generalised).

Learner: every rank of a torchrun world holds the DeepSeek-V4.1 base (experts EP-sharded over the
world when ``--ep-size`` > 1, dense weights FSDP2-sharded) with frozen weights and trainable
query-LoRA adapters (``attention.q_a`` of the selected layers). Rollouts come from a service that
speaks the LoRA RPC protocol (``rollout.remote``): the reference's vLLM service or this library's
``rollout.native_service``; rank 0 owns the client and every host call runs through
``rank_zero_call``, which broadcasts 5 s heartbeats so peers never sit in one long collective.

Per group of G responses to one prompt: rewards -> group advantages (constant groups are skipped)
-> ``train_group`` (responses scored in planner micro-batches; clipped GRPO, or decoupled
Token-TIS against the native-old policy that generated the group; loss / G; one AdamW step on the
adapters) -> export the adapters as a LoRA packet -> activate on the service (the ack must match)
-> resume. With prefetch, the next group is sampled while the current one trains (policy lag 1,
allowed only with the adapter snapshot of the generating policy). Evaluation runs before and after
on a held-out set; ``summary.json``, ``groups.jsonl`` and ``updates.jsonl`` record the run.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import math
import os
import time
import uuid
from concurrent.futures import ThreadPoolExecutor, wait
from contextlib import contextmanager
from datetime import timedelta
from pathlib import Path

import torch
import torch.distributed as dist

from .algorithm import decoupled_token_tis_loss, group_advantages, grpo_loss, response_log_probs, response_log_probs_batch
from .learner_batch_planner import parse_learner_batch_shapes, plan_learner_microbatches, plan_response_ownership
from .lora_config import SUPPORTED_LORA_RANKS, DistributedLoRAConfig, parse_lora_layers
from .lora_export import export_q_a_update


def rank_zero_call(function):
    """Run ``function`` on rank 0; all ranks receive its result (or its error) with heartbeats."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return function()
    executor = ThreadPoolExecutor(max_workers=1) if dist.get_rank() == 0 else None
    future = executor.submit(function) if executor is not None else None
    try:
        while True:
            box = [None]
            if future is not None:
                wait([future], timeout=5)
                if not future.done():
                    box[0] = {"heartbeat": True}
                else:
                    try:
                        box[0] = {"result": future.result()}
                    except BaseException as error:
                        box[0] = {"error_type": type(error).__name__, "error": str(error)}
            dist.broadcast_object_list(box, src=0)
            if box[0].get("heartbeat"):
                continue
            if "error" in box[0]:
                raise RuntimeError(f"rank-zero operation failed: {box[0]['error_type']}: {box[0]['error']}")
            return box[0]["result"]
    finally:
        if executor is not None:
            executor.shutdown(wait=True)


def request_specs(record, *, count, phase, index, seed, max_tokens, temperature, lineage):
    return [{"prompt_ids": record.prompt_ids, "max_tokens": max_tokens, "temperature": temperature,
             "sampling_seed": seed + index * 32 + s,
             "request_id": hashlib.sha256(f"{lineage}:{phase}:{index}:{s}".encode()).hexdigest()[:32]}
            for s in range(count)]


def validate_results(results, record, ack, count):
    if not isinstance(results, list) or len(results) != count:
        raise ValueError("only complete rollout groups may enter the learner")
    for r in results:
        actions, old = r["action_token_ids"], r["behavior_log_probs"]
        ok = (r["context_token_ids"] == record.prompt_ids and actions and len(actions) == len(old)
              and all(type(t) is int and t >= 0 for t in actions) and all(math.isfinite(p) and p <= 1e-6 for p in old)
              and r.get("logprob_convention") == "sampled_distribution"
              and r["generation_metrics"]["policy_ack"] == ack and r["finish_reason"] in {"eos", "stop", "length"}
              and r["stop_token_count"] in (0, 1))
        if not ok:
            raise ValueError("rollout tokens, sampled probabilities, or policy identity differ")
    return results


def sample_record(client, record, *, count, phase, index, args, lineage, temperature=None, max_tokens=None):
    ack = dict(client.ack)
    specs = request_specs(record, count=count, phase=phase, index=index, seed=args.seed,
                          max_tokens=max_tokens or args.max_new_tokens,
                          temperature=args.temperature if temperature is None else temperature, lineage=lineage)
    results = validate_results(client.sample_group(specs), record, ack, count)
    for spec, r in zip(specs, results):
        if (r["generation_metrics"].get("request_id") != spec["request_id"]
                or r["generation_metrics"].get("sampling_seed") != spec["sampling_seed"]):
            raise ValueError("rollout response order or sampling identity differs")
    return results


def score_rewards(results, record, reward):
    values = []
    for r in results:
        ids, stop = r["action_token_ids"], r["stop_token_count"]
        values.append(float(reward(record, ids[:-stop] if stop else ids)))
    return values


def evaluate(client, records, reward, args, lineage, phase) -> dict:
    ack, correct, tokens, started = dict(client.ack), 0.0, 0, time.monotonic()
    for start in range(0, len(records), 32):
        batch = records[start:start + 32]
        specs = [request_specs(rec, count=1, phase=phase, index=start + i, seed=args.seed,
                               max_tokens=args.max_new_tokens, temperature=args.eval_temperature, lineage=lineage)[0]
                 for i, rec in enumerate(batch)]
        results = client.sample_group(specs)
        for rec, r in zip(batch, results):
            validate_results([r], rec, ack, 1)
            correct += score_rewards([r], rec, reward)[0]
            tokens += len(r["action_token_ids"])
    ids = json.dumps([rec.prompt_ids for rec in records], separators=(",", ":"))
    return {"n": len(records), "reward_sum": correct, "reward_mean": correct / len(records), "output_tokens": tokens,
            "elapsed_seconds": time.monotonic() - started, "temperature": args.eval_temperature, "policy_ack": ack,
            "ordered_ids_sha256": hashlib.sha256(ids.encode()).hexdigest()}


def adapter_parameters(optimizer):
    return [p for g in optimizer.param_groups for p in g["params"]]


def adapter_snapshot(optimizer):
    local = [(p.to_local() if hasattr(p, "to_local") else p) for p in adapter_parameters(optimizer)]
    return [t.detach().clone() for t in local]


@contextmanager
def adapter_parameters_at(optimizer, values):
    """Temporarily score with other adapter values (the native-old policy), then restore."""
    params = adapter_parameters(optimizer)
    locals_ = [(p.to_local() if hasattr(p, "to_local") else p) for p in params]
    saved = [t.detach().clone() for t in locals_]
    try:
        with torch.no_grad():
            for t, v in zip(locals_, values):
                t.copy_(v)
        yield
    finally:
        with torch.no_grad():
            for t, v in zip(locals_, saved):
                t.copy_(v)


def gradient_norm(optimizer) -> float:
    sq = None
    for p in adapter_parameters(optimizer):
        if p.grad is None:
            continue
        g = p.grad.to_local() if hasattr(p.grad, "to_local") else p.grad
        v = g.float().square().sum()
        sq = v if sq is None else sq + v
    if sq is None:
        return 0.0
    if dist.is_initialized() and any(hasattr(p, "device_mesh") for p in adapter_parameters(optimizer)):
        dist.all_reduce(sq)
    return float(sq.sqrt())


def train_group(model, optimizer, results, advantages, args, update, *, expected_ack=None, native_old=None) -> dict:
    """Sum of per-response losses / G in planner micro-batches, then one adapter update."""
    g = len(results)
    correction = args.rollout_correction
    if len(advantages) != g or not bool(torch.isfinite(torch.as_tensor(advantages)).all()):
        raise ValueError("a learner update requires every response and finite advantages")
    generating = results[0]["generation_metrics"]["policy_ack"]
    lag = None
    if expected_ack is not None:
        if (expected_ack["version"] != update - 1 or generating.get("lineage") != expected_ack["lineage"]
                or any(r["generation_metrics"]["policy_ack"] != generating for r in results)):
            raise ValueError("generating and learner policy receipts disagree")
        lag = expected_ack["version"] - generating["version"]
        if not 0 <= lag <= (0 if args.disable_prefetch else 1) or (lag == 0 and generating != expected_ack):
            raise ValueError("generating policy has an invalid policy lag")
        if correction == "none" and lag:
            raise ValueError("a lagged group needs decoupled Token-TIS")
    lengths = [len(r["context_token_ids"]) + len(r["action_token_ids"]) - 1 for r in results]
    if args.learner_response_ownership == "sharded":
        plan = plan_response_ownership(lengths, dist.get_rank(), dist.get_world_size())
    else:
        plan = plan_learner_microbatches(lengths, args.learner_microbatch_size,
                                         parse_learner_batch_shapes(args.learner_batch_shapes))
    optimizer.zero_grad(set_to_none=True)
    metrics = [None] * g
    for planned in plan:
        idx = planned["response_indices"]
        batch = [results[i] for i in idx]
        prompts = [r["context_token_ids"] for r in batch]
        responses = [r["action_token_ids"] for r in batch]

        def score():
            if len(batch) == 1:
                return [response_log_probs(model, prompts[0], responses[0], args.temperature)]
            return response_log_probs_batch(model, prompts, responses, args.temperature)

        old = None
        if correction == "decoupled-token-tis":
            with torch.no_grad():
                if lag:
                    with adapter_parameters_at(optimizer, native_old):
                        old = [v.detach().clone() for v in score()]
                else:
                    old = [v.detach().clone() for v in score()]
        current = score()
        losses = []
        for j, i in enumerate(idx):
            placeholder = planned.get("is_placeholder", False)
            adv = 0.0 if placeholder else float(advantages[i])
            if correction == "decoupled-token-tis":
                loss, row = decoupled_token_tis_loss([current[j]], [old[j]], [batch[j]["behavior_log_probs"]], [adv],
                                                     clip_eps=args.clip_eps, is_cap=args.rollout_is_cap)
            else:
                loss, row = grpo_loss([current[j]], [batch[j]["behavior_log_probs"]], [adv], clip_eps=args.clip_eps,
                                      kl_beta=0.0)
            losses.append(loss * 0 if placeholder else loss)
            if not placeholder:
                metrics[i] = row
        (torch.stack(losses).sum() / g).backward()
    if args.learner_response_ownership == "sharded":
        parts = [None] * dist.get_world_size()
        dist.all_gather_object(parts, [(i, r) for i, r in enumerate(metrics) if r is not None])
        metrics = [None] * g
        for part in parts:
            for i, r in part:
                metrics[i] = r
        # each rank holds the gradient of its own responses only: sum them
        for p in adapter_parameters(optimizer):
            if p.grad is not None and not hasattr(p.grad, "to_local"):
                dist.all_reduce(p.grad)
    norm = gradient_norm(optimizer)
    if not math.isfinite(norm) or norm <= 0:
        raise ValueError("a genuine optimizer update requires finite nonzero adapter gradients")
    before = adapter_snapshot(optimizer)
    optimizer.step()
    changed = sum(int((a != b.to(a.device)).sum()) for a, b in
                  zip([(p.to_local() if hasattr(p, "to_local") else p).detach() for p in adapter_parameters(optimizer)],
                      before))
    pooled = {k: sum(r[k] for r in metrics) / g for k in metrics[0] if isinstance(metrics[0][k], (int, float))}
    return {**pooled, "rollout_correction": correction, "policy_lag": lag, "gradient_norm": norm,
            "changed_adapter_elements": changed, "microbatches": len(plan)}


def load_learner(args, lora_config: DistributedLoRAConfig, device):
    """Base weights (frozen), query adapters (trainable), EP + FSDP2 across the world."""
    from ..lora import inject_lora
    from ..models.dsv4.checkpoint import load_dsv41_backbone_prefix
    from ..models.dsv4.config import DeepSeekV41Config
    from ..parallel.cp import ContextParallel
    from ..parallel.dispatch import TokenDispatcher

    cfg = DeepSeekV41Config.from_json(Path(args.model_dir) / "config.json")
    world = dist.get_world_size() if dist.is_initialized() else 1
    meshes, dispatcher = None, TokenDispatcher()
    if world > 1:
        from ..parallel.meshes import ParallelMeshes

        meshes = ParallelMeshes.build(ep=args.learner_ep_size, device_type=device.type, engram=True)
        if meshes.ep is not None:
            from ..parallel.dispatch import AllToAllTokenDispatcher

            dispatcher = AllToAllTokenDispatcher(meshes.ep)
    dtype = torch.bfloat16 if device.type == "cuda" else torch.float32
    # score with the values the rollout service's FP8 / FP4 KV cache returns (reference
    # dsv41_train/rl/native_lora.py:208 loads its scoring model with cache_quantization="hf")
    model = load_dsv41_backbone_prefix(args.model_dir, num_layers=cfg.num_hidden_layers, device=device, dtype=dtype,
                                       context_parallel=ContextParallel(), token_dispatcher=dispatcher,
                                       engram_mesh=meshes.engram if meshes is not None else None,
                                       cache_quantization=args.cache_quantization)
    for p in model.parameters():
        p.requires_grad_(False)
    for layer in lora_config.selected_layers(cfg.num_hidden_layers):
        inject_lora(model.model.layers[layer], lora_config.lora_config())
        q_a = model.model.layers[layer].attention.q_a
        q_a.lora_a.data = q_a.lora_a.data.to(torch.bfloat16)
        q_a.lora_b.data = q_a.lora_b.data.to(torch.bfloat16)
    for layer in model.model.layers:
        if layer.attention.indexer is not None:
            layer.attention.indexer.stable_topk = True
    if meshes is not None:
        from ..parallel.fsdp import apply_fsdp

        apply_fsdp(model, meshes, param_dtype=dtype)
    model.distributed_lora_config = lora_config
    params = [p for p in model.parameters() if p.requires_grad]
    optimizer = torch.optim.AdamW(params, lr=args.learning_rate, weight_decay=0.0, foreach=False)
    return model, optimizer


def load_records(args, tokenizer):
    from .data import build_reward, load_jsonl

    if args.dataset == "gsm8k":
        from .gsm8k import prepare_data

        train, test, reward, provenance = prepare_data(args.train_jsonl, args.test_jsonl, tokenizer,
                                                       revision=args.dataset_revision, seed=args.seed,
                                                       max_prompt_tokens=args.max_prompt_tokens,
                                                       max_train_groups=args.max_groups,
                                                       eval_questions=args.eval_questions)
        return train, test, reward, provenance
    train = load_jsonl(args.train_jsonl, tokenizer=tokenizer, max_prompt_tokens=args.max_prompt_tokens)[:args.max_groups]
    test = load_jsonl(args.test_jsonl, tokenizer=tokenizer, max_prompt_tokens=args.max_prompt_tokens)[:args.eval_questions]
    return train, test, build_reward(args.reward, tokenizer=tokenizer), {"train": str(args.train_jsonl)}


def run(args) -> dict:
    from ..rollout.lora_transport import policy_ack
    from ..rollout.remote import RemoteLoRAClient
    from .tokenizer import ModelTokenizer

    if args.rollout_correction not in {"none", "decoupled-token-tis"}:
        raise ValueError("unknown rollout correction mode")
    if args.learner_response_ownership == "sharded" and (args.group_size != 32 or args.learner_microbatch_size != 4):
        raise ValueError("sharded response ownership requires G32 and micro-batch 4")
    lora_config = DistributedLoRAConfig(args.lora_rank, args.lora_alpha, args.lora_layers)
    token = os.environ["DSV41_ROLLOUT_TOKEN"]
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if torch.cuda.is_available() and args.device != "cpu":
        torch.cuda.set_device(local_rank)
        device = torch.device("cuda", local_rank)
        backend = "nccl"
    else:
        device, backend = torch.device("cpu"), "gloo"
    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29520")
        os.environ.setdefault("RANK", "0")
        os.environ.setdefault("WORLD_SIZE", "1")
        dist.init_process_group(backend, timeout=timedelta(seconds=600))
    rank = dist.get_rank()
    output = Path(args.output_dir).resolve()
    summary = {"status": "started", "optimizer_updates": 0, "adapter_configuration": lora_config.to_dict()}
    client = executor = None
    started = time.monotonic()
    try:
        tokenizer = ModelTokenizer(args.model_dir)
        train, test, reward, data = load_records(args, tokenizer)
        rank_zero_call(lambda: output.mkdir(parents=True, exist_ok=False))
        identity = {k: hashlib.sha256((Path(args.model_dir) / n).read_bytes()).hexdigest()
                    for k, n in (("config_sha256", "config.json"), ("index_sha256", "model.safetensors.index.json"))}
        lineage = rank_zero_call(lambda: "grpo-" + uuid.uuid4().hex)
        if rank == 0:
            client = RemoteLoRAClient(args.rollout_host, args.rollout_port, token, timeout=args.rpc_timeout)
            executor = ThreadPoolExecutor(max_workers=1)
        startup = rank_zero_call(lambda: client.initialize(lora_config=lora_config.to_dict()))
        if startup["base_identity"] != identity:
            raise ValueError("rollout and learner mounted base identities differ")
        model, optimizer = load_learner(args, lora_config, device)

        def activate(version):
            packet = export_q_a_update(model, version=version, lineage=lineage, adapter_id=version + 1,
                                       base_identity=identity, optimizer=optimizer)

            def send():
                receipt = client.activate(*packet)
                if receipt["ack"] != policy_ack(packet[0]):
                    raise ValueError("service activation acknowledgement differs from the learner packet")
                client.resume()
                return receipt["ack"]

            return rank_zero_call(send)

        ack = activate(0)
        snapshots = {0: adapter_snapshot(optimizer)}
        summary["baseline"] = rank_zero_call(lambda: evaluate(client, test, reward, args, lineage, "baseline"))
        pending = None
        for gi, record in enumerate(train):
            results = rank_zero_call(lambda: pending.result() if pending is not None else sample_record(
                client, record, count=args.group_size, phase="train", index=gi, args=args, lineage=lineage))
            rewards = score_rewards(results, record, reward)
            adv = group_advantages(rewards)
            usable = bool(adv.abs().sum())
            row = {"group": gi, "behavior_version": results[0]["generation_metrics"]["policy_ack"]["version"],
                   "reward_sum": sum(rewards), "responses": len(results), "usable": usable}
            if rank == 0:
                with (output / "groups.jsonl").open("a") as f:
                    f.write(json.dumps(row) + "\n")
            pending = None
            if not usable:
                continue
            update = summary["optimizer_updates"] + 1
            if (not args.disable_prefetch and rank == 0 and update > 1 and gi + 1 < len(train)
                    and update < args.updates):
                nxt = train[gi + 1]
                pending = executor.submit(sample_record, client, nxt, count=args.group_size, phase="train",
                                          index=gi + 1, args=args, lineage=lineage)
            metrics = train_group(model, optimizer, results, adv, args, update, expected_ack=ack,
                                  native_old=snapshots.get(row["behavior_version"]))
            summary["optimizer_updates"] = update
            rank_zero_call(lambda: pending.result() if pending is not None else None)  # join before pausing
            rank_zero_call(lambda: client.pause())
            ack = activate(update)
            snapshots[update] = adapter_snapshot(optimizer)
            snapshots = {v: s for v, s in snapshots.items() if v >= update - 1}
            if rank == 0:
                with (output / "updates.jsonl").open("a") as f:
                    f.write(json.dumps({"update": update, "group": gi, "policy_ack": ack, **metrics}) + "\n")
            if update >= args.updates:
                break
        if summary["optimizer_updates"] < args.updates:
            raise RuntimeError("available nonconstant groups did not complete the requested updates")
        summary["final"] = rank_zero_call(lambda: evaluate(client, test, reward, args, lineage, "final"))
        summary.update(status="completed", policy_ack=ack, data=data)
    except BaseException as error:
        summary.update(status="failed", error_type=type(error).__name__, reason=str(error))
        raise
    finally:
        if executor is not None:
            executor.shutdown(wait=True, cancel_futures=True)
        if client is not None:
            try:
                client.close()
            except Exception:
                pass
        summary["elapsed_seconds"] = time.monotonic() - started
        if rank == 0 and output.is_dir():
            (output / "summary.json").write_text(json.dumps(summary, indent=2, sort_keys=True, allow_nan=False) + "\n")
    return summary


def parse_args(argv=None):
    p = argparse.ArgumentParser(description="Distributed query-LoRA GRPO against a LoRA rollout service")
    for name in ("model-dir", "train-jsonl", "test-jsonl", "output-dir"):
        p.add_argument("--" + name, required=True)
    p.add_argument("--rollout-host", default="127.0.0.1")
    p.add_argument("--rollout-port", type=int, required=True)
    p.add_argument("--rpc-timeout", type=float, default=7200)
    p.add_argument("--dataset", choices=("jsonl", "gsm8k"), default="jsonl")
    p.add_argument("--dataset-revision", default=None)
    p.add_argument("--reward", default="numeric_answer")
    p.add_argument("--rollout-correction", choices=("none", "decoupled-token-tis"), default="none")
    p.add_argument("--rollout-is-cap", type=float, default=2.0)
    p.add_argument("--disable-prefetch", action="store_true")
    p.add_argument("--updates", type=int, default=3)
    p.add_argument("--max-groups", type=int, default=64)
    p.add_argument("--eval-questions", type=int, default=128)
    p.add_argument("--group-size", type=int, default=32)
    p.add_argument("--learner-microbatch-size", type=int, default=4)
    p.add_argument("--learner-response-ownership", choices=("replicated", "sharded"), default="replicated")
    p.add_argument("--learner-ep-size", type=int, default=1)
    p.add_argument("--learner-batch-shapes", default=None)
    p.add_argument("--lora-rank", type=int, choices=SUPPORTED_LORA_RANKS, default=8)
    p.add_argument("--lora-alpha", type=float, default=8.0)
    p.add_argument("--lora-layers", type=parse_lora_layers, default=None)
    p.add_argument("--cache-quantization", choices=("hf", "none"), default="hf",
                   help="hf: score under the rollout engine's FP8 window-KV / FP4 compressed-KV and indexer cache")
    p.add_argument("--seed", type=int, default=42)
    p.add_argument("--max-prompt-tokens", type=int, default=256)
    p.add_argument("--max-new-tokens", type=int, default=256)
    p.add_argument("--temperature", type=float, default=0.8)
    p.add_argument("--eval-temperature", type=float, default=0.01)
    p.add_argument("--learning-rate", type=float, default=1e-4)
    p.add_argument("--clip-eps", type=float, default=0.2)
    p.add_argument("--device", default="auto")
    return p.parse_args(argv)


def main(argv=None) -> None:
    try:
        run(parse_args(argv))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
