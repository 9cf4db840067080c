"""Fixed-prompt evaluation of a policy and the inspectable per-sample rows.

Row and metric fields follow ``dsv41_train/rl/evaluation.py:14-76`` (the evaluation files are read
by the same analysis scripts). Evaluation draws ``eval_samples_per_prompt`` samples per prompt
from a CPU generator seeded with ``eval_seed``, so two evaluations of one policy agree exactly.
"""

from __future__ import annotations

import json
from pathlib import Path
from statistics import mean, pstdev

import torch

from .rollout import generate_group


def append_jsonl(path, rows) -> None:
    target = Path(path)
    target.parent.mkdir(parents=True, exist_ok=True)
    lines = [json.dumps(row, ensure_ascii=False, allow_nan=False) for row in rows]
    with target.open("a", encoding="utf-8") as handle:
        handle.writelines(line + "\n" for line in lines)


def decoded_fields(tokenizer, ids, name, *, skip_special_tokens=True) -> dict:
    """``{name}_text``; ids without text (padded vocabularies) give None and ``{name}_decode_error``."""
    try:
        text = tokenizer.decode(ids, skip_special_tokens=skip_special_tokens)
    except ValueError as error:
        return {f"{name}_text": None, f"{name}_decode_error": str(error)}
    return {f"{name}_text": text}


def sample_record(record, sample, *, step, group_id, tokenizer=None, phase="train") -> dict:
    row = {"phase": phase, "step": step, "group_id": group_id, "policy_version": sample.policy_version,
           "prompt_ids": sample.prompt_ids, "response_ids": sample.response_ids, "reward": sample.reward,
           "raw_reward": sample.raw_reward, "finish_reason": sample.finish_reason,
           "stop_token_count": sample.stop_token_count, "metadata": record.metadata}
    if tokenizer is not None:
        row |= decoded_fields(tokenizer, sample.prompt_ids, "prompt", skip_special_tokens=False)
        row |= decoded_fields(tokenizer, sample.content_ids, "response")
    return row


def evaluation_metrics(samples, records, *, step, phase) -> dict:
    rewards = [s.reward for s in samples]
    return {
        "event": "eval", "phase": phase, "step": step, "policy_version": step, "prompts": len(records),
        "samples": len(samples), "reward_mean": mean(rewards), "reward_std": pstdev(rewards),
        "raw_reward_mean": mean(s.raw_reward for s in samples),
        "response_length_mean": mean(len(s.response_ids) for s in samples),
        "truncation_fraction": mean(s.finish_reason == "length" for s in samples),
        "zero_reward_fraction": mean(r == 0 for r in rewards),
    }


def evaluate_policy(model, records, config, *, reward_fn, generation_kwargs, step, tokenizer=None, output_dir=None,
                    phase="eval", return_rows=False):
    if not records:
        raise ValueError("evaluation requires at least one prompt")
    generator = torch.Generator(device="cpu").manual_seed(config.eval_seed)
    samples, rows = [], []
    for group_id, record in enumerate(records):
        group = generate_group(model, record, group_size=config.eval_samples_per_prompt,
                               max_new_tokens=config.max_new_tokens, temperature=config.temperature,
                               policy_version=step, group_id=group_id, generator=generator, reward_fn=reward_fn,
                               **generation_kwargs)
        for sample in group.samples:
            samples.append(sample)
            rows.append(sample_record(record, sample, step=step, group_id=group_id, tokenizer=tokenizer, phase=phase))
    metrics = evaluation_metrics(samples, records, step=step, phase=phase)
    if output_dir is not None:
        out = Path(output_dir)
        append_jsonl(out / "eval-samples.jsonl", rows)
        append_jsonl(out / "eval-metrics.jsonl", [metrics])
    return (metrics, rows) if return_rows else metrics


__all__ = ["append_jsonl", "decoded_fields", "evaluate_policy", "evaluation_metrics", "sample_record"]
