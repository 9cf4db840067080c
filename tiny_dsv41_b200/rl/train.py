"""``python -m tiny_dsv41_b200.rl.train``: local GRPO with the rollout manager
(flags of ``dsv41_train/rl/train.py:11-66``)."""

from __future__ import annotations

import argparse
import json
from pathlib import Path

from .config import RLConfig
from .runtime import run_training


def main(argv=None) -> None:
    parser = argparse.ArgumentParser(description="GRPO with a rollout-manager child process and a native learner")
    parser.add_argument("--model-dir", required=True, help="checkpoint directory; the family comes from config.json")
    parser.add_argument("--data", required=True, help="JSONL with prompt, messages or prompt_ids")
    parser.add_argument("--eval-data", help="independent validation JSONL; enables baseline and periodic evaluation")
    parser.add_argument("--config", required=True, help="RL runtime JSON")
    parser.add_argument("--random-init", "--allow-random-init", action="store_true",
                        help="initialize from config.json without loading base weights")
    parser.add_argument("--resume", help="step-XXXXXXXX.pt checkpoint")
    parser.add_argument("--max-steps", type=int, help="total optimizer steps, including restored steps")
    parser.add_argument("--output-dir", help="checkpoint and log directory")
    parser.add_argument("--trainer-num-gpus", type=int, help="trainer GPU count; zero selects CPU")
    parser.add_argument("--rollout-num-gpus", type=int, help="rollout GPU count; allocated after trainer GPUs")
    parser.add_argument("--rollout-engine", choices=("vllm", "native-pytorch"))
    parser.add_argument("--trainable-scope", choices=("all", "lm_head", "lora"))
    parser.add_argument("--initial-adapter", help="portable SFT adapter; requires trainable-scope=lora")
    parser.add_argument("--optimizer", choices=("adamw", "sgd"))
    parser.add_argument("--engram-offload", action=argparse.BooleanOptionalAction, default=None)
    parser.add_argument("--gradient-checkpointing", action=argparse.BooleanOptionalAction, default=None)
    args = parser.parse_args(argv)
    values = json.loads(Path(args.config).read_text(encoding="utf-8"))
    values["rollout_engine"] = args.rollout_engine or values.get("rollout_engine", "vllm")
    for name in ("max_steps", "output_dir", "trainable_scope", "initial_adapter", "optimizer", "engram_offload",
                 "gradient_checkpointing"):
        if getattr(args, name) is not None:
            values[name] = getattr(args, name)
    if args.trainer_num_gpus is not None or args.rollout_num_gpus is not None:
        if args.trainer_num_gpus is None or args.rollout_num_gpus is None:
            parser.error("specify both --trainer-num-gpus and --rollout-num-gpus")
        values.pop("learner_devices", None)
        values.pop("rollout_devices", None)
        values.update(trainer_num_gpus=args.trainer_num_gpus, rollout_num_gpus=args.rollout_num_gpus)
    checkpoint = run_training(model_dir=args.model_dir, data_path=args.data, config=RLConfig.from_dict(values),
                              random_init=args.random_init, resume=args.resume, eval_data_path=args.eval_data)
    print(f"checkpoint: {checkpoint}", flush=True)


if __name__ == "__main__":
    main()
