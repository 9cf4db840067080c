"""``python -m tiny_dsv41_b200.rollout``: inspect / validate / plan / run prompt-response rollouts
(the prompt-response part of the reference's ``rollout-manager`` CLI, ``rollout_manager/cli.py``).

    inspect  --tasks T.jsonl                 task count and prompt-length range
    validate --tasks T.jsonl --model-dir M   every record is valid for the model's vocabulary
    plan     --tasks T.jsonl --group-size G  the episode identities a run would execute
    run      --tasks T.jsonl --model-dir M --output-dir O [--random-init] [--group-size G]
             executes every plan through the coordinator; events, results and summary under O
"""

from __future__ import annotations

import argparse
import asyncio
import hashlib
import json
import uuid
from pathlib import Path

from .contracts import EpisodeIdentity, EpisodePlan, ResourceRequirements, TaskSpec


def load_tasks(path) -> list[TaskSpec]:
    from ..rl.data import PromptRecord

    tasks = []
    for i, line in enumerate(Path(path).read_text().splitlines()):
        if not line.strip():
            continue
        raw = json.loads(line)
        record = PromptRecord.from_mapping(raw)
        body = {"prompt_ids": record.prompt_ids, "target_ids": record.target_ids, "metadata": record.metadata}
        source = hashlib.sha256(json.dumps(body, sort_keys=True, separators=(",", ":")).encode()).hexdigest()
        tasks.append(TaskSpec("prompt-response", f"prompt-response/{i}", source,
                              {"prompt_response": {"record": body, "group_id": i}},
                              ResourceRequirements("pytorch-policy", accounting="backend-stage")))
    if not tasks:
        raise ValueError("the task file holds no records")
    return tasks


def plan_episodes(tasks, group_size: int, run_id: str, seed: int = 0) -> list[EpisodePlan]:
    return [EpisodePlan(EpisodeIdentity(run_id, t.benchmark, t.task_id, str(g), s, sampling_seed=seed + g * 1000 + s),
                        t, None) for g, t in enumerate(tasks) for s in range(group_size)]


def main(argv=None) -> None:
    p = argparse.ArgumentParser(prog="python -m tiny_dsv41_b200.rollout", description="prompt-response rollouts")
    sub = p.add_subparsers(dest="command", required=True)
    for name in ("inspect", "validate", "plan", "run"):
        s = sub.add_parser(name)
        s.add_argument("--tasks", required=True)
        if name in ("validate", "run"):
            s.add_argument("--model-dir", required=True)
        if name in ("plan", "run"):
            s.add_argument("--group-size", type=int, default=4)
            s.add_argument("--seed", type=int, default=0)
        if name == "run":
            s.add_argument("--output-dir", required=True)
            s.add_argument("--random-init", action="store_true")
            s.add_argument("--max-new-tokens", type=int, default=16)
            s.add_argument("--temperature", type=float, default=1.0)
            s.add_argument("--reward", default="token_accuracy")
            s.add_argument("--workers", type=int, default=1)
    args = p.parse_args(argv)
    tasks = load_tasks(args.tasks)
    if args.command == "inspect":
        lengths = [len(t.payload["prompt_response"]["record"]["prompt_ids"]) for t in tasks]
        print(json.dumps({"tasks": len(tasks), "prompt_tokens_min": min(lengths), "prompt_tokens_max": max(lengths)}))
        return
    if args.command == "plan":
        plans = plan_episodes(tasks, args.group_size, "plan", args.seed)
        print(json.dumps([{"task_id": x.identity.task_id, "group_id": x.identity.group_id,
                           "sample_index": x.identity.sample_index, "sampling_seed": x.identity.sampling_seed}
                          for x in plans]))
        return
    from ..rl.family import load_model_config

    config = load_model_config(args.model_dir)
    bad = [t.task_id for t in tasks if any(tok >= config.vocab_size for tok in t.payload["prompt_response"]["record"]["prompt_ids"])]
    if bad:
        raise SystemExit(f"records with token ids outside the vocabulary: {bad[:5]}")
    if args.command == "validate":
        print(json.dumps({"tasks": len(tasks), "valid": True}))
        return
    import torch

    from ..rl.config import RLConfig
    from ..rl.data import build_reward
    from ..rl.runtime import make_model
    from .backends import PromptResponseBackend
    from .coordinator import Coordinator
    from .events import EventStore

    cfg = RLConfig.from_dict({"rollout_engine": "native-pytorch", "seed": args.seed})
    model = make_model(args.model_dir, config, cfg, ("cpu",), args.random_init, role="actor").eval()
    backend = PromptResponseBackend(model, build_reward(args.reward), max_new_tokens=args.max_new_tokens,
                                    temperature=args.temperature)
    run_id = uuid.uuid4().hex
    store = EventStore(Path(args.output_dir), run_id)
    coordinator = Coordinator({"prompt-response": backend}, max_workers=args.workers, event_store=store)
    plans = plan_episodes(tasks, args.group_size, run_id, args.seed)
    with torch.inference_mode():
        results = asyncio.run(coordinator.run_wave(plans))
    rewards = [r.native_outcome["reward"] for r in results if r.score_eligible]
    summary = {"episodes": len(results), "eligible": len(rewards),
               "reward_mean": sum(rewards) / len(rewards) if rewards else None,
               "quarantined_workers": coordinator.quarantined}
    store.write_summary(summary)
    store.close()
    print(json.dumps(summary))


__all__ = ["load_tasks", "main", "plan_episodes"]
