"""``python -m tiny_dsv41_b200.rl.train`` (also ``python -m dsv41_train.rl.train``): local GRPO with
a rollout-manager child process and this library's learner.

The flags are the command-line interface of ``dsv41_train/rl/train.py:11-66``: a JSON run config
plus command-line overrides of some of its fields.
"""

from __future__ import annotations

import argparse
import json
from pathlib import Path

from .config import RLConfig
from .runtime import run_training

# flags that override the run config's field of the same name when given
_OVERRIDES = ("max_steps", "output_dir", "trainable_scope", "initial_adapter", "optimizer", "engram_offload",
              "gradient_checkpointing")


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="GRPO: a rollout manager samples, the learner trains")
    p.add_argument("--model-dir", required=True, help="model directory; config.json names the family")
    p.add_argument("--data", required=True, help="training prompts (JSONL with prompt, messages or prompt_ids)")
    p.add_argument("--eval-data", help="held-out prompts (JSONL); enables the baseline and periodic evaluation")
    p.add_argument("--config", required=True, help="RL run configuration (JSON)")
    p.add_argument("--random-init", "--allow-random-init", action="store_true",
                   help="build the model from config.json without loading weights")
    p.add_argument("--resume", help="continue from a step-XXXXXXXX.pt checkpoint")
    p.add_argument("--max-steps", type=int, help="total optimizer steps, restored steps included")
    p.add_argument("--output-dir", help="where checkpoints and logs go")
    p.add_argument("--trainer-num-gpus", type=int, help="learner GPUs (0 = CPU)")
    p.add_argument("--rollout-num-gpus", type=int, help="sampler GPUs, numbered after the learner's")
    p.add_argument("--rollout-engine", choices=("vllm", "native-pytorch"))
    p.add_argument("--trainable-scope", choices=("all", "lm_head", "lora"))
    p.add_argument("--initial-adapter", help="adapter exported by SFT (needs --trainable-scope lora)")
    p.add_argument("--optimizer", choices=("adamw", "sgd"))
    p.add_argument("--engram-offload", action=argparse.BooleanOptionalAction, default=None)
    p.add_argument("--gradient-checkpointing", action=argparse.BooleanOptionalAction, default=None)
    return p


def config_values(args, parser: argparse.ArgumentParser) -> dict:
    values = json.loads(Path(args.config).read_text(encoding="utf-8"))
    values["rollout_engine"] = args.rollout_engine or values.get("rollout_engine", "vllm")
    values.update({name: getattr(args, name) for name in _OVERRIDES if getattr(args, name) is not None})
    counts = (args.trainer_num_gpus, args.rollout_num_gpus)
    if counts != (None, None):
        if None in counts:
            parser.error("specify both --trainer-num-gpus and --rollout-num-gpus")
        for name in ("learner_devices", "rollout_devices"):  # the counts replace explicit lists
            values.pop(name, None)
        values["trainer_num_gpus"], values["rollout_num_gpus"] = counts
    return values


def main(argv=None) -> None:
    parser = build_parser()
    args = parser.parse_args(argv)
    config = RLConfig.from_dict(config_values(args, parser))
    checkpoint = run_training(model_dir=args.model_dir, data_path=args.data, config=config,
                              random_init=args.random_init, resume=args.resume, eval_data_path=args.eval_data)
    print(f"checkpoint: {checkpoint}", flush=True)


if __name__ == "__main__":
    main()
