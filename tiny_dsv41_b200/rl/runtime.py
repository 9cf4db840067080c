"""Local GRPO runtime: a learner loop that trains on groups sampled by a rollout-manager child.

Behaviour kept from ``dsv41_train/rl/runtime.py`` (``run_training``, ``train_groups``): the
checks on data, devices, reward and resume; the exclusive output directory; publishing policy
version v before the manager may sample with it; dropping groups whose policy lag exceeds
``max_policy_lag``; one optimizer step per ``groups_per_step`` groups with gradient clipping; and
after every step commit -> publish -> checkpoint -> activate -> resume, so a crash between any two
of these resumes from the checkpoint. Every stage is timed in ``learner-stage-timings.jsonl``.

Structure here: :class:`_Session` owns the run (inputs, models, manager, counters) and has one
method per phase of a step; :func:`run_training` opens the output directory lock and drives it.
The vLLM rollout engine is an external service: this runtime samples with the native engine and
refuses ``rollout_engine = "vllm"`` unless a provider factory is passed in.
"""

from __future__ import annotations

import fcntl
import json
import os
import queue
import time
import uuid
from contextlib import contextmanager
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


def make_model(model_dir, model_config, config, devices, random_init, *, role="learner"):
    """The policy (or frozen reference, or rollout copy) with this run's trainable scope."""
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
    """Versions between the learner and a group's sampling policy; None when beyond ``maximum``."""
    lag = learner_version - rollout_version
    if lag < 0:
        raise ValueError("rollout policy version is newer than learner")
    return None if lag > maximum else lag


def validate_device_ownership(learner_devices, rollout_devices) -> None:
    def gpus(devices):
        return {torch.device(d).index for d in devices if torch.device(d).type == "cuda"}

    if gpus(learner_devices) & gpus(rollout_devices):
        raise ValueError("learner and rollout CUDA devices must have separate ownership")


class _StepTotals:
    """Running sums of one optimizer step's GRPO metrics (each sample weighted 1 / samples)."""

    def __init__(self, samples: int, groups: int) -> None:
        self.samples, self.groups = samples, groups
        self.values: dict[str, float] = {}
        self.rewards: list[float] = []
        self.nonzero = self.zero_variance = self.truncated = 0

    def add_group(self, advantages: torch.Tensor) -> None:
        live = int(advantages.count_nonzero())
        self.nonzero += live
        self.zero_variance += int(live == 0)

    def add_sample(self, sample, values: dict) -> None:
        for name, value in values.items():
            self.values[name] = self.values.get(name, 0.0) + value / self.samples
        self.rewards.append(sample.reward)
        self.truncated += int(sample.finish_reason == "length")

    def result(self, grad_norm: float) -> dict:
        out = dict(self.values)
        out.update(reward_mean=sum(self.rewards) / len(self.rewards), grad_norm=grad_norm,
                   nonzero_advantages=self.nonzero, samples=self.samples,
                   zero_variance_group_fraction=self.zero_variance / self.groups,
                   truncation_fraction=self.truncated / self.samples, optimizer_step_applied=True)
        return out


def train_groups(model, reference, optimizer, groups, config) -> dict:
    """One optimizer step over ``groups``: per sample, backward of the clipped GRPO loss divided by
    the number of samples (group-normalised advantages, optional KL to ``reference``); then the
    gradient norm is clipped (a non-finite norm aborts before the step) and the optimizer steps."""
    model.train()
    optimizer.zero_grad(set_to_none=True)
    totals = _StepTotals(sum(len(g.samples) for g in groups), len(groups))
    for group in groups:
        advantages = group_advantages([s.reward for s in group.samples])
        totals.add_group(advantages)
        for sample, advantage in zip(group.samples, advantages):
            current = response_log_probs(model, sample.prompt_ids, sample.response_ids, config.temperature)
            anchor = None
            if reference is not None:
                with torch.no_grad():
                    anchor = [response_log_probs(reference, sample.prompt_ids, sample.response_ids,
                                                 config.temperature)]
            loss, values = grpo_loss([current], [sample.behavior_log_probs], [float(advantage)],
                                     clip_eps=config.clip_eps, ref_log_probs=anchor, kl_beta=config.kl_beta)
            if not torch.isfinite(loss):
                raise FloatingPointError("non-finite RL loss; optimizer step was not applied")
            (loss / totals.samples).backward()
            totals.add_sample(sample, values)
    trainable = [p for p in model.parameters() if p.requires_grad]
    norm = torch.nn.utils.clip_grad_norm_(trainable, config.max_grad_norm, error_if_nonfinite=True, foreach=False)
    optimizer.step()
    model.assert_invariants()
    return totals.result(float(norm))


def prepare_records(data_path, model_config, config, tokenizer):
    """Prompt records that fit the context with ``max_new_tokens`` to spare, ids in the vocabulary."""
    room = model_config.max_position_embeddings - config.max_new_tokens
    if config.max_prompt_tokens is not None:
        room = min(room, config.max_prompt_tokens)
    if room < 1:
        raise ValueError("max_new_tokens must leave room for a prompt within the model context")
    records = load_jsonl(data_path, tokenizer=tokenizer, max_prompt_tokens=room, length_policy=config.length_policy)
    for record in records:
        if len(record.prompt_ids) + config.max_new_tokens > model_config.max_position_embeddings:
            raise ValueError("prompt length + max_new_tokens exceeds model context length")
        ids = [*record.prompt_ids, *(record.target_ids or [])]
        if ids and max(ids) >= model_config.vocab_size:
            raise ValueError("dataset token IDs must be inside the model vocabulary")
    return records


def validate_reward_records(records, reward, spec) -> None:
    """Target-based rewards need targets; text rewards are tried once on an empty response."""
    from .rewards import TEXT_REWARDS

    for index, record in enumerate(records):
        if spec in {"token_accuracy", "exact_match"} and record.target_ids is None:
            raise ValueError(f"record {index}: reward {spec} requires target_ids")
        if spec not in TEXT_REWARDS:
            continue
        try:
            reward(record, [])
        except (TypeError, ValueError) as exc:
            raise ValueError(f"record {index}: {exc}") from exc


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


@contextmanager
def exclusive_output(output_dir: Path):
    """Hold an advisory lock on ``output_dir/.run.lock`` for the run; a second run fails fast."""
    handle = (output_dir / ".run.lock").open("a+", encoding="utf-8")
    try:
        fcntl.flock(handle, fcntl.LOCK_EX | fcntl.LOCK_NB)
    except BlockingIOError:
        handle.close()
        raise RuntimeError(f"another training process owns output_dir: {output_dir}") from None
    try:
        yield
    finally:
        fcntl.flock(handle, fcntl.LOCK_UN)
        handle.close()


def _make_optimizer(model, config):
    trainable = [p for p in model.parameters() if p.requires_grad]
    kind = torch.optim.SGD if config.optimizer == "sgd" else torch.optim.AdamW
    return kind(trainable, lr=config.learning_rate, weight_decay=config.weight_decay, foreach=False)


class _Session:
    """One GRPO run: inputs, learner (and reference) model, optimizer, rollout manager, counters."""

    def __init__(self, *, model_dir, data_path, config: RLConfig, random_init, resume, eval_data_path,
                 rollout_factory) -> None:
        self.model_dir = str(Path(model_dir).resolve())
        self.data_path = str(Path(data_path).resolve())
        self.config, self.random_init, self.resume = config, random_init, resume
        self.rollout_factory = rollout_factory
        self.model_config = load_model_config(self.model_dir)
        for devices in (config.learner_devices, config.rollout_devices):
            layer_device_map(self.model_config.num_hidden_layers, devices)
            validate_available_devices(devices)
        validate_device_ownership(config.learner_devices, config.rollout_devices)
        has_tokenizer = (Path(self.model_dir) / "tokenizer.json").is_file()
        self.tokenizer = ModelTokenizer(self.model_dir) if has_tokenizer else None
        self.records = prepare_records(self.data_path, self.model_config, config, self.tokenizer)
        self.eval_records = (prepare_records(eval_data_path, self.model_config, config, self.tokenizer)
                             if eval_data_path else [])
        train_prompts = {tuple(r.prompt_ids) for r in self.records}
        if any(tuple(r.prompt_ids) in train_prompts for r in self.eval_records):
            raise ValueError("validation prompts overlap training prompts; use an independent validation set")
        self.reward_fn = build_reward(config.reward, tokenizer=self.tokenizer)
        validate_reward_records(self.records + self.eval_records, self.reward_fn, config.reward)
        self.identity = self._identity(eval_data_path)
        self.output_dir = Path(config.output_dir).resolve()
        self.sampling = {"temperature": config.temperature, "top_p": 1, "top_k": 0}
        self.manager = None
        self.step = self.next_group_id = self.dropped = 0
        self.rng_state = self.recovery = None
        self.lineage = uuid.uuid4().hex
        self.ack = None
        self.previous_train = None

    def _identity(self, eval_data_path) -> dict:
        config = self.config
        identity = run_identity(self.model_dir, self.data_path, self.random_init, eval_data_path=eval_data_path)
        identity["trainable_scope"] = config.trainable_scope
        if config.initial_sft_checkpoint is not None:
            from .family import initial_sft_source

            identity["initial_sft_checkpoint"] = initial_sft_source(self.model_dir, self.model_config, config,
                                                                    self.random_init).identity
        if config.trainable_scope == "lora":
            identity["lora"] = {"rank": config.lora_rank, "alpha": config.lora_alpha,
                                "targets": list(policy_lora_config(config, self.model_config).targets)}
        return identity

    # -- setup ----------------------------------------------------------------------------------
    def build(self, timings: StageTimings) -> None:
        cfg = self.config
        self.model = timings.call("model_startup", make_model, self.model_dir, self.model_config, cfg,
                                  cfg.learner_devices, self.random_init, details={"devices": list(cfg.learner_devices)})
        self.reference = None
        if cfg.kl_beta:
            self.reference = timings.call("reference_model_startup", make_model, self.model_dir, self.model_config,
                                          cfg, cfg.learner_devices, self.random_init, role="reference")
            self.reference.eval().requires_grad_(False)
        self.optimizer = _make_optimizer(self.model, cfg)
        if self.resume:
            state = timings.call("checkpoint_restore", load_training_checkpoint, self.resume, self.model,
                                 self.optimizer, cfg, self.identity)
            self.step, self.next_group_id = state["step"], state["next_group_id"]
            self.rng_state, self.dropped = state["rollout_rng_state"], state["dropped_groups"]
            self.recovery = state.get("manager_state")
            if self.recovery is not None:
                self.lineage = self.recovery["active_policy"]["lineage"]
        elif any(self.output_dir.glob("step-*.pt")):
            raise FileExistsError("output_dir already has checkpoints; use --resume or a new output directory")
        self.generation = generation_options(self.model_dir, self.model_config, cfg)
        self.config = replace(cfg, eos_token_ids=tuple(self.generation["eos_token_id"]))
        if self.step >= self.config.max_steps:
            raise ValueError("max_steps must exceed the restored checkpoint step")
        if any(int(p.stem.removeprefix("step-")) > self.step for p in self.output_dir.glob("step-*.pt")):
            raise FileExistsError("output_dir contains later checkpoints; resume into a new --output-dir")

    def evaluate(self, timings: StageTimings, stage: str, phase: str | None = None) -> None:
        extra = {} if phase is None else {"phase": phase}
        metrics = timings.call(stage, evaluate_policy, self.model, self.eval_records, self.config,
                               reward_fn=self.reward_fn, generation_kwargs=self.generation, step=self.step,
                               tokenizer=self.tokenizer, output_dir=self.output_dir, **extra)
        print(json.dumps(metrics, sort_keys=True, allow_nan=False), flush=True)

    def publish(self, timings: StageTimings, stage: str) -> dict:
        return timings.call(stage, publish_policy_artifact, self.model, self.step, self.output_dir / "policies",
                            lineage=self.lineage, identity=self.identity, sampling=self.sampling,
                            details={"policy_version": self.step})

    def start_manager(self, timings: StageTimings) -> None:
        from .manager import RolloutManager

        artifact = self.publish(timings, "initial_policy_publish")
        with timings.interval("manager_startup", policy_version=self.step):
            factory = self.rollout_factory or RolloutManager
            self.manager = factory(self.model_dir, self.model_config, self.config, self.records, self.random_init,
                                   initial_policy=artifact, recovery_state=self.recovery,
                                   next_group_id=self.next_group_id, rng_state=self.rng_state,
                                   event_root=self.output_dir / f"rollouts-{uuid.uuid4().hex}")
            self.ack = self.manager.start()
            validate_policy_ack(self.ack, artifact)
        cfg = self.config
        print(json.dumps({"event": "started", "learner_pid": os.getpid(), "rollout_pid": self.manager.pid,
                          "policy_ack": self.ack, "rollout_engine": "native-pytorch",
                          "engram_device": self.model.engram_device, "trainer_devices": list(cfg.learner_devices),
                          "rollout_devices": list(cfg.rollout_devices), "policy_version": self.step}), flush=True)

    # -- one step -------------------------------------------------------------------------------
    def collect(self, timings: StageTimings):
        """``groups_per_step`` groups trainable at this policy version (stale or excluded ones are
        committed as dropped on the way)."""
        cfg = self.config
        groups, packets, lags = [], [], []
        deadline = time.monotonic() + cfg.worker_timeout_seconds
        with timings.interval("wait_eligible_groups", step=self.step, required_groups=cfg.groups_per_step):
            while len(groups) < cfg.groups_per_step:
                if time.monotonic() > deadline:
                    raise TimeoutError("timed out waiting for a fresh rollout group")
                try:
                    packet = self.manager.get(timeout=0.2)
                except queue.Empty:
                    continue
                admitted = admit_packet(packet, self.step, cfg, self.manager, self.output_dir)
                if admitted is None:
                    self.dropped += 1
                    continue
                groups.append(admitted[0])
                lags.append(admitted[1])
                packets.append(packet)
        return groups, packets, lags

    def train(self, timings: StageTimings, groups):
        timings.call("actor_pause_before_training", self.manager.pause, details={"step": self.step})
        with timings.interval("train_groups", step=self.step + 1):
            begin = time.monotonic()
            metrics = train_groups(self.model, self.reference, self.optimizer, groups, self.config)
            span = (begin, time.monotonic())
        self.step += 1
        return metrics, span

    def commit_publish_activate(self, timings: StageTimings, groups) -> dict:
        """Retire the groups, publish policy v(step), checkpoint, then hand the policy to the manager."""
        self.manager.commit(consumed_group_ids=[g.group_id for g in groups])
        self.recovery = timings.call("actor_pause_after_group_commit", self.manager.pause, details={"step": self.step})
        self.next_group_id, self.rng_state = self.recovery["next_group_id"], self.recovery["rng_state"]
        artifact = self.publish(timings, "policy_publish")
        path = self.output_dir / f"step-{self.step:08d}.pt"
        timings.call("checkpoint_write", save_training_checkpoint, path, self.model, self.optimizer, step=self.step,
                     config=self.config, identity=self.identity, next_group_id=self.next_group_id,
                     rollout_rng_state=self.rng_state, dropped_groups=self.dropped, manager_state=self.recovery,
                     policy_publication={**artifact, "state": "staged", "previous_ack": self.ack},
                     details={"step": self.step, "checkpoint": str(path)})
        with timings.interval("actor_activation", policy_version=self.step):
            self.ack = self.manager.activate(artifact)
            validate_policy_ack(self.ack, artifact)
        timings.call("actor_resume", self.manager.resume, details={"policy_version": self.step})
        return artifact

    def log_samples(self, groups) -> None:
        limit = self.config.log_samples_per_step
        if not limit:
            return
        rows = [sample_record(self.records[g.group_id % len(self.records)], sample, step=self.step,
                              group_id=g.group_id, tokenizer=self.tokenizer)
                for g in groups for sample in g.samples][:limit]
        append_jsonl(self.output_dir / "train-samples.jsonl", rows)

    def log_metrics(self, metrics, artifact, groups, packets, lags, span) -> None:
        overlap = 0.0  # sampling time of this step's groups that ran during the previous update
        if self.previous_train is not None:
            lo, hi = self.previous_train
            overlap = sum(max(0.0, min(p["finished_at"], hi) - max(p["started_at"], lo)) for p in packets)
        metrics.update(event="train", step=self.step, policy_version=self.step, policy_lag_max=max(lags),
                       policy_digest=artifact["digest"], policy_ack=self.ack, dropped_groups=self.dropped,
                       next_group_id=self.next_group_id, rollout_versions=[g.policy_version for g in groups],
                       train_seconds=span[1] - span[0], overlap_previous_train_seconds=overlap)
        line = json.dumps(metrics, sort_keys=True, allow_nan=False)
        print(line, flush=True)
        with (self.output_dir / "metrics.jsonl").open("a", encoding="utf-8") as f:
            f.write(line + "\n")
        self.previous_train = span

    def due_for_evaluation(self) -> bool:
        cfg = self.config
        return bool(self.eval_records) and (self.step % (cfg.eval_interval or cfg.checkpoint_interval) == 0
                                            or self.step == cfg.max_steps)


def run_training(*, model_dir, data_path, config: RLConfig, random_init=False, resume=None, eval_data_path=None,
                 rollout_factory=None):
    """Train until ``config.max_steps``; returns the last checkpoint's path."""
    config.validate()
    if config.checkpoint_interval != 1:
        raise ValueError("manager training requires checkpoint_interval=1 before policy activation")
    if config.rollout_engine == "vllm" and rollout_factory is None:
        raise ValueError("the vLLM rollout engine is an external service: pass its provider, or select "
                         "rollout_engine=native-pytorch")
    torch.set_num_threads(config.num_threads)
    run = _Session(model_dir=model_dir, data_path=data_path, config=config, random_init=random_init, resume=resume,
                   eval_data_path=eval_data_path, rollout_factory=rollout_factory)
    run.output_dir.mkdir(parents=True, exist_ok=True)
    with exclusive_output(run.output_dir):
        timings = StageTimings(run.output_dir / "learner-stage-timings.jsonl",
                               clock_domain="learner_process_monotonic")
        try:
            run.build(timings)
            if run.eval_records:
                run.evaluate(timings, "baseline_evaluation", phase="resume" if resume else "baseline")
            run.start_manager(timings)
            while run.step < run.config.max_steps:
                groups, packets, lags = run.collect(timings)
                metrics, span = run.train(timings, groups)
                artifact = run.commit_publish_activate(timings, groups)
                run.log_samples(groups)
                run.log_metrics(metrics, artifact, groups, packets, lags, span)
                if run.due_for_evaluation():
                    run.evaluate(timings, "evaluation")
            return run.output_dir / f"step-{run.step:08d}.pt"
        finally:
            if run.manager is not None:
                timings.call("manager_close", run.manager.close)


__all__ = ["admit_packet", "exclusive_output", "make_model", "policy_lag", "prepare_records", "run_training",
           "train_groups", "validate_device_ownership", "validate_reward_records"]
