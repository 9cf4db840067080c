"""Local GRPO runtime: learner loop over a rollout-manager child process.

Flow of ``dsv41_train/rl/runtime.py:299-590`` (``run_training``) and ``:175-262``
(``train_groups``):

  validate config -> prompts / reward -> run identity -> output-dir lock (fcntl) -> learner policy
  (+ frozen reference when kl_beta > 0) -> optimizer -> resume or fresh -> publish policy v0 ->
  start manager (ack must name v0) -> loop { wait groups_per_step eligible groups (stale groups
  beyond max_policy_lag are dropped and committed as such) -> pause -> train_groups -> commit ->
  publish policy v(step) -> checkpoint step-XXXXXXXX.pt -> activate (ack checked) -> resume ->
  metrics / samples / eval } -> close manager.

``train_groups`` accumulates, for each sample, (clipped GRPO loss * fraction) / samples, clips the
gradient norm (non-finite norms abort before the optimizer step) and steps the optimizer once.
Every stage is recorded in ``learner-stage-timings.jsonl``.

The vLLM rollout engine is an external service; this runtime samples with the native engine
(``rollout_engine = "native-pytorch"``) and refuses ``vllm`` unless a provider is passed in.
"""

from __future__ import annotations

import fcntl
import json
import os
import queue
import time
import uuid
from dataclasses import replace
from pathlib import Path

import torch

from ..utils.stage_timings import StageTimings
from .algorithm import group_advantages, grpo_loss, response_log_probs
from .checkpoint import (load_training_checkpoint, publish_policy_artifact, run_identity, save_training_checkpoint,
                         validate_policy_ack)
from .config import RLConfig
from .data import build_reward, load_jsonl
from .evaluation import append_jsonl, evaluate_policy, sample_record
from .family import build_policy, load_model_config, policy_lora_config
from .parallel import layer_device_map, validate_available_devices
from .rollout import generation_options
from .tokenizer import ModelTokenizer


def make_model(model_dir, model_config, config: RLConfig, devices, random_init, *, role="learner"):
    from ..train.sft_export import resolve_initial_bundle
    from .family import initial_sft_source

    config = resolve_initial_bundle(config)
    torch.manual_seed(config.seed)
    model = build_policy(model_dir, model_config, random_init=random_init, devices=devices,
                         dtype=getattr(torch, config.dtype), trainable_scope=config.trainable_scope,
                         lora_config=policy_lora_config(config, model_config), initial_adapter=config.initial_adapter,
                         engram_offload=config.engram_offload,
                         sft_source=initial_sft_source(model_dir, model_config, config, random_init))
    if getattr(model_config, "model_type", None) == "qwen3_moe":
        model.qwen_last_position_only = config.qwen_last_position_only
        model.qwen_kv_cache = config.qwen_kv_cache
    if config.gradient_checkpointing:
        model.backend.gradient_checkpointing_enable()
    return model


def policy_lag(learner_version: int, rollout_version: int, maximum: int):
    lag = learner_version - rollout_version
    if lag < 0:
        raise ValueError("rollout policy version is newer than learner")
    return lag if lag <= maximum else None


def validate_device_ownership(learner_devices, rollout_devices) -> None:
    def cuda(devices):
        return {torch.device(d).index for d in devices if torch.device(d).type == "cuda"}

    if cuda(learner_devices) & cuda(rollout_devices):
        raise ValueError("learner and rollout CUDA devices must have separate ownership")


def train_groups(model, reference, optimizer, groups, config) -> dict:
    model.train()
    optimizer.zero_grad(set_to_none=True)
    total = sum(len(g.samples) for g in groups)
    metrics: dict = {}
    rewards, nonzero, zero_var, truncated = [], 0, 0, 0
    for group in groups:
        advantages = group_advantages([s.reward for s in group.samples])
        nonzero += int(advantages.count_nonzero())
        zero_var += int(not bool(advantages.count_nonzero()))
        for sample, advantage in zip(group.samples, advantages):
            current = response_log_probs(model, sample.prompt_ids, sample.response_ids, config.temperature)
            ref = None
            if reference is not None:
                with torch.no_grad():
                    ref = response_log_probs(reference, sample.prompt_ids, sample.response_ids, config.temperature)
            loss, values = grpo_loss([current], [sample.behavior_log_probs], [float(advantage)],
                                     clip_eps=config.clip_eps, ref_log_probs=[ref] if ref is not None else None,
                                     kl_beta=config.kl_beta)
            if not torch.isfinite(loss):
                raise FloatingPointError("non-finite RL loss; optimizer step was not applied")
            (loss / total).backward()
            for name, value in values.items():
                metrics[name] = metrics.get(name, 0.0) + value / total
            rewards.append(sample.reward)
            truncated += int(sample.finish_reason == "length")
    params = [p for p in model.parameters() if p.requires_grad]
    norm = torch.nn.utils.clip_grad_norm_(params, config.max_grad_norm, error_if_nonfinite=True, foreach=False)
    optimizer.step()
    model.assert_invariants()
    metrics.update(reward_mean=sum(rewards) / len(rewards), grad_norm=float(norm), nonzero_advantages=nonzero,
                   samples=total, zero_variance_group_fraction=zero_var / len(groups),
                   truncation_fraction=truncated / total, optimizer_step_applied=True)
    return metrics


def _check_inputs(records, model_config, config) -> None:
    for record in records:
        if len(record.prompt_ids) + config.max_new_tokens > model_config.max_position_embeddings:
            raise ValueError("prompt length + max_new_tokens exceeds model context length")
        if any(t >= model_config.vocab_size for t in list(record.prompt_ids) + list(record.target_ids or [])):
            raise ValueError("dataset token IDs must be inside the model vocabulary")


def prepare_records(data_path, model_config, config, tokenizer):
    limit = model_config.max_position_embeddings - config.max_new_tokens
    if config.max_prompt_tokens is not None:
        limit = min(limit, config.max_prompt_tokens)
    if limit < 1:
        raise ValueError("max_new_tokens must leave room for a prompt within the model context")
    records = load_jsonl(data_path, tokenizer=tokenizer, max_prompt_tokens=limit, length_policy=config.length_policy)
    _check_inputs(records, model_config, config)
    return records


def validate_reward_records(records, reward, spec) -> None:
    from .rewards import TEXT_REWARDS

    for index, record in enumerate(records):
        if spec in {"token_accuracy", "exact_match"} and record.target_ids is None:
            raise ValueError(f"record {index}: reward {spec} requires target_ids")
        if spec in TEXT_REWARDS:
            try:
                reward(record, [])
            except (TypeError, ValueError) as exc:
                raise ValueError(f"record {index}: {exc}") from exc


def _optimizer(model, config):
    params = [p for p in model.parameters() if p.requires_grad]
    if config.optimizer == "sgd":
        return torch.optim.SGD(params, lr=config.learning_rate, weight_decay=config.weight_decay, foreach=False)
    return torch.optim.AdamW(params, lr=config.learning_rate, weight_decay=config.weight_decay, foreach=False)


def admit_packet(packet: dict, step: int, config, manager, output_dir: Path):
    """One rollout packet: (group, policy lag) when it is trainable now, or None after committing it
    as dropped (a provider's exclusion, logged to ``excluded-groups.jsonl``, or a group whose policy
    lag exceeds ``max_policy_lag``). A group of the wrong size is an error."""
    if packet.get("exclusion") is not None:
        manager.commit(dropped_group_ids=[packet["group_id"]])
        append_jsonl(output_dir / "excluded-groups.jsonl", [packet["exclusion"]])
        return None
    group = packet["group"]
    lag = policy_lag(step, group.policy_version, config.max_policy_lag)
    if lag is None:
        manager.commit(dropped_group_ids=[group.group_id])
        return None
    if len(group.samples) != config.group_size:
        raise ValueError("incomplete group")
    return group, lag


def run_training(*, model_dir, data_path, config: RLConfig, random_init=False, resume=None, eval_data_path=None,
                 rollout_factory=None):
    config.validate()
    if config.checkpoint_interval != 1:
        raise ValueError("manager training requires checkpoint_interval=1 before policy activation")
    if config.rollout_engine == "vllm" and rollout_factory is None:
        raise ValueError("the vLLM rollout engine is an external service: pass its provider, or select "
                         "rollout_engine=native-pytorch")
    torch.set_num_threads(config.num_threads)
    model_dir, data_path = str(Path(model_dir).resolve()), str(Path(data_path).resolve())
    model_config = load_model_config(model_dir)
    for devices in (config.learner_devices, config.rollout_devices):
        layer_device_map(model_config.num_hidden_layers, devices)
        validate_available_devices(devices)
    validate_device_ownership(config.learner_devices, config.rollout_devices)
    tokenizer = ModelTokenizer(model_dir) if (Path(model_dir) / "tokenizer.json").is_file() else None
    records = prepare_records(data_path, model_config, config, tokenizer)
    eval_records = prepare_records(eval_data_path, model_config, config, tokenizer) if eval_data_path else []
    if {tuple(r.prompt_ids) for r in records} & {tuple(r.prompt_ids) for r in eval_records}:
        raise ValueError("validation prompts overlap training prompts; use an independent validation set")
    reward_fn = build_reward(config.reward, tokenizer=tokenizer)
    validate_reward_records(records + eval_records, reward_fn, config.reward)
    identity = run_identity(model_dir, data_path, random_init, eval_data_path=eval_data_path)
    identity["trainable_scope"] = config.trainable_scope
    if config.initial_sft_checkpoint is not None:
        from .family import initial_sft_source

        identity["initial_sft_checkpoint"] = initial_sft_source(model_dir, model_config, config, random_init).identity
    if config.trainable_scope == "lora":
        identity["lora"] = {"rank": config.lora_rank, "alpha": config.lora_alpha,
                            "targets": list(policy_lora_config(config, model_config).targets)}
    output_dir = Path(config.output_dir).resolve()
    output_dir.mkdir(parents=True, exist_ok=True)
    lock_handle = (output_dir / ".run.lock").open("a+", encoding="utf-8")
    try:
        fcntl.flock(lock_handle, fcntl.LOCK_EX | fcntl.LOCK_NB)
    except BlockingIOError:
        lock_handle.close()
        raise RuntimeError(f"another training process owns output_dir: {output_dir}") from None
    manager = None
    timings = StageTimings(output_dir / "learner-stage-timings.jsonl", clock_domain="learner_process_monotonic")
    try:
        model = timings.call("model_startup", make_model, model_dir, model_config, config, config.learner_devices,
                             random_init, details={"devices": list(config.learner_devices)})
        reference = None
        if config.kl_beta:
            reference = timings.call("reference_model_startup", make_model, model_dir, model_config, config,
                                     config.learner_devices, random_init, role="reference")
            reference.eval().requires_grad_(False)
        optimizer = _optimizer(model, config)
        step, next_group_id, rng_state, dropped, recovery = 0, 0, None, 0, None
        lineage = uuid.uuid4().hex
        if resume:
            state = timings.call("checkpoint_restore", load_training_checkpoint, resume, model, optimizer, config,
                                 identity)
            step, next_group_id = state["step"], state["next_group_id"]
            rng_state, dropped = state["rollout_rng_state"], state["dropped_groups"]
            recovery = state.get("manager_state")
            if recovery is not None:
                lineage = recovery["active_policy"]["lineage"]
            del state
        elif any(output_dir.glob("step-*.pt")):
            raise FileExistsError("output_dir already has checkpoints; use --resume or a new output directory")
        generation = generation_options(model_dir, model_config, config)
        config = replace(config, eos_token_ids=tuple(generation["eos_token_id"]))
        if step >= config.max_steps:
            raise ValueError("max_steps must exceed the restored checkpoint step")
        if any(int(p.stem.removeprefix("step-")) > step for p in output_dir.glob("step-*.pt")):
            raise FileExistsError("output_dir contains later checkpoints; resume into a new --output-dir")
        if eval_records:
            metrics = timings.call("baseline_evaluation", evaluate_policy, model, eval_records, config,
                                   reward_fn=reward_fn, generation_kwargs=generation, step=step, tokenizer=tokenizer,
                                   output_dir=output_dir, phase="resume" if resume else "baseline")
            print(json.dumps(metrics, sort_keys=True, allow_nan=False), flush=True)
        from .manager import RolloutManager

        sampling = {"temperature": config.temperature, "top_p": 1, "top_k": 0}
        artifact = timings.call("initial_policy_publish", publish_policy_artifact, model, step, output_dir / "policies",
                                lineage=lineage, identity=identity, sampling=sampling, details={"policy_version": step})
        with timings.interval("manager_startup", policy_version=step):
            manager = (rollout_factory or RolloutManager)(
                model_dir, model_config, config, records, random_init, initial_policy=artifact,
                recovery_state=recovery, next_group_id=next_group_id, rng_state=rng_state,
                event_root=output_dir / f"rollouts-{uuid.uuid4().hex}")
            ack = manager.start()
            validate_policy_ack(ack, artifact)
        print(json.dumps({"event": "started", "learner_pid": os.getpid(), "rollout_pid": manager.pid,
                          "policy_ack": ack, "rollout_engine": "native-pytorch",
                          "engram_device": model.engram_device, "trainer_devices": list(config.learner_devices),
                          "rollout_devices": list(config.rollout_devices), "policy_version": step}), flush=True)
        previous_train = None
        while step < config.max_steps:
            groups, packets, lags = [], [], []
            deadline = time.monotonic() + config.worker_timeout_seconds
            with timings.interval("wait_eligible_groups", step=step, required_groups=config.groups_per_step):
                while len(groups) < config.groups_per_step:
                    if time.monotonic() > deadline:
                        raise TimeoutError("timed out waiting for a fresh rollout group")
                    try:
                        packet = manager.get(timeout=0.2)
                    except queue.Empty:
                        continue
                    admitted = admit_packet(packet, step, config, manager, output_dir)
                    if admitted is None:
                        dropped += 1
                        continue
                    group, lag = admitted
                    groups.append(group)
                    packets.append(packet)
                    lags.append(lag)
            timings.call("actor_pause_before_training", manager.pause, details={"step": step})
            with timings.interval("train_groups", step=step + 1):
                train_start = time.monotonic()
                metrics = train_groups(model, reference, optimizer, groups, config)
                train_end = time.monotonic()
            step += 1
            manager.commit(consumed_group_ids=[g.group_id for g in groups])
            recovery = timings.call("actor_pause_after_group_commit", manager.pause, details={"step": step})
            next_group_id, rng_state = recovery["next_group_id"], recovery["rng_state"]
            artifact = timings.call("policy_publish", publish_policy_artifact, model, step, output_dir / "policies",
                                    lineage=lineage, identity=identity, sampling=sampling,
                                    details={"policy_version": step})
            checkpoint = output_dir / f"step-{step:08d}.pt"
            timings.call("checkpoint_write", save_training_checkpoint, checkpoint, model, optimizer, step=step,
                         config=config, identity=identity, next_group_id=next_group_id, rollout_rng_state=rng_state,
                         dropped_groups=dropped, manager_state=recovery,
                         policy_publication={**artifact, "state": "staged", "previous_ack": ack},
                         details={"step": step, "checkpoint": str(checkpoint)})
            with timings.interval("actor_activation", policy_version=step):
                ack = manager.activate(artifact)
                validate_policy_ack(ack, artifact)
            timings.call("actor_resume", manager.resume, details={"policy_version": step})
            if config.log_samples_per_step:
                rows = []
                for group in groups:
                    record = records[group.group_id % len(records)]
                    for sample in group.samples:
                        if len(rows) < config.log_samples_per_step:
                            rows.append(sample_record(record, sample, step=step, group_id=group.group_id,
                                                      tokenizer=tokenizer))
                append_jsonl(output_dir / "train-samples.jsonl", rows)
            overlap = 0.0
            if previous_train is not None:
                start, end = previous_train
                overlap = sum(max(0.0, min(p["finished_at"], end) - max(p["started_at"], start)) for p in packets)
            metrics.update(event="train", step=step, policy_version=step, policy_lag_max=max(lags),
                           policy_digest=artifact["digest"], policy_ack=ack, dropped_groups=dropped,
                           next_group_id=next_group_id, rollout_versions=[g.policy_version for g in groups],
                           train_seconds=train_end - train_start, overlap_previous_train_seconds=overlap)
            line = json.dumps(metrics, sort_keys=True, allow_nan=False)
            print(line, flush=True)
            with (output_dir / "metrics.jsonl").open("a", encoding="utf-8") as f:
                f.write(line + "\n")
            previous_train = (train_start, train_end)
            if eval_records and (step % (config.eval_interval or config.checkpoint_interval) == 0
                                 or step == config.max_steps):
                metrics = timings.call("evaluation", evaluate_policy, model, eval_records, config, reward_fn=reward_fn,
                                       generation_kwargs=generation, step=step, tokenizer=tokenizer,
                                       output_dir=output_dir)
                print(json.dumps(metrics, sort_keys=True, allow_nan=False), flush=True)
        return output_dir / f"step-{step:08d}.pt"
    finally:
        try:
            if manager is not None:
                timings.call("manager_close", manager.close)
        finally:
            fcntl.flock(lock_handle, fcntl.LOCK_UN)
            lock_handle.close()


__all__ = ["make_model", "policy_lag", "prepare_records", "run_training", "train_groups",
           "validate_device_ownership"]
