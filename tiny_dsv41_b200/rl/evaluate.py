"""``python -m tiny_dsv41_b200.rl.evaluate`` (also ``python -m dsv41_train.rl.evaluate``): score a
saved RL policy on a JSONL prompt set without training. Flags follow
``dsv41_train/rl/evaluate.py:16-44``."""

from __future__ import annotations

import argparse
import json
from dataclasses import replace
from pathlib import Path

from .data import build_reward
from .evaluation import evaluate_policy
from .rollout import generation_options
from .runtime import prepare_records, validate_reward_records
from .sample import load_checkpoint_model
from .tokenizer import ModelTokenizer


def _parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="Score a saved RL policy on text or token-ID prompts")
    for flag in ("--model-dir", "--checkpoint", "--data", "--output-dir"):
        p.add_argument(flag, required=True)
    p.add_argument("--devices", default="cpu", help="cpu, or CUDA devices separated by commas")
    p.add_argument("--reward", help="reward spec (default: the checkpoint's)")
    p.add_argument("--max-new-tokens", type=int)
    p.add_argument("--seed", type=int, help="sampling seed (default: the checkpoint's eval_seed)")
    return p


def main(argv=None) -> None:
    args = _parser().parse_args(argv)
    devices = tuple(d.strip() for d in args.devices.split(","))
    model, config, step, _ = load_checkpoint_model(model_dir=args.model_dir, checkpoint=args.checkpoint,
                                                   devices=devices, max_new_tokens=args.max_new_tokens)
    overrides = {"reward": args.reward or config.reward}
    if args.seed is not None:
        overrides["eval_seed"] = args.seed
    config = replace(config, **overrides)
    config.validate()
    has_tokenizer = (Path(args.model_dir) / "tokenizer.json").is_file()
    tokenizer = ModelTokenizer(args.model_dir) if has_tokenizer else None
    records = prepare_records(args.data, model.config, config, tokenizer)
    reward = build_reward(config.reward, tokenizer=tokenizer)
    validate_reward_records(records, reward, config.reward)
    options = generation_options(args.model_dir, model.config, config)
    metrics = evaluate_policy(model, records, config, tokenizer=tokenizer, reward_fn=reward,
                              generation_kwargs=options, step=step, output_dir=args.output_dir)
    print(json.dumps(metrics, sort_keys=True, allow_nan=False), flush=True)


if __name__ == "__main__":
    main()
