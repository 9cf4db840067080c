"""``python -m tiny_dsv41_b200.rl.sample``: generate from an RL checkpoint and its base model
(``dsv41_train/rl/sample.py:21-153``: same flags and output fields).

The checkpoint's base identity (config hash, base weight files, text assets) must match the
mounted model directory; no training data is needed. The policy state is restored onto a freshly
built model; ``--seed`` only seeds the CPU sampling generator.
"""

from __future__ import annotations

import argparse
import json
from dataclasses import replace
from pathlib import Path
from typing import Optional, Sequence

import torch

from .checkpoint import load_policy, run_identity
from .config import RLConfig
from .data import PromptRecord
from .evaluation import decoded_fields
from .family import load_model_config
from .rollout import generate_group, generation_options
from .runtime import make_model
from .tokenizer import ModelTokenizer

_BASE_KEYS = ("config_sha256", "random_init", "weights", "text_assets")


def load_checkpoint_model(*, model_dir, checkpoint, devices: Sequence[str] = ("cpu",),
                          max_new_tokens: Optional[int] = None, temperature: Optional[float] = None,
                          seed: Optional[int] = None):
    model_dir = Path(model_dir).resolve()
    state = torch.load(checkpoint, map_location="cpu", weights_only=False)
    if not isinstance(state, dict) or state.get("format_version") not in (1, 2):
        raise ValueError("unsupported RL checkpoint format")
    if not all(k in state for k in ("config", "identity", "policy", "step")):
        raise ValueError("RL checkpoint is missing config, identity, policy or step")
    identity = state["identity"]
    if not isinstance(identity, dict) or type(identity.get("random_init")) is not bool:
        raise ValueError("checkpoint identity must contain a boolean random_init flag")
    random_init = identity["random_init"]
    current = run_identity(model_dir, None, random_init)
    if {k: identity.get(k) for k in _BASE_KEYS} != {k: current.get(k) for k in _BASE_KEYS}:
        raise ValueError("checkpoint base-model identity differs from the mounted model directory")
    version = state["step"]
    if type(version) is not int or version < 0:
        raise ValueError("checkpoint step must be a nonnegative integer")
    values = dict(state["config"])
    values.update(learner_devices=tuple(devices), rollout_devices=tuple(devices), rollout_engine="native-pytorch")
    if max_new_tokens is not None:
        values["max_new_tokens"] = max_new_tokens
    if temperature is not None:
        values["temperature"] = temperature
    config = RLConfig.from_dict(values)
    sampling_seed = config.seed if seed is None else seed
    if type(sampling_seed) is not int or not 0 <= sampling_seed < 2 ** 63 - 1:
        raise ValueError("sampling seed must be an integer in [0, 2**63 - 1)")
    torch.set_num_threads(config.num_threads)
    model_config = load_model_config(model_dir)
    model = make_model(model_dir, model_config, config, devices, random_init, role="actor")
    load_policy(model, state["policy"])
    model.eval()
    return model, config, version, sampling_seed


def sample_checkpoint(*, model_dir, checkpoint, prompt_ids=None, prompt=None, messages=None, devices=("cpu",),
                      max_new_tokens=None, temperature=None, seed=None) -> dict:
    tokenizer = ModelTokenizer(model_dir) if (Path(model_dir) / "tokenizer.json").is_file() else None
    value = {k: v for k, v in (("prompt_ids", prompt_ids), ("prompt", prompt), ("messages", messages)) if v is not None}
    record = PromptRecord.from_mapping(value, tokenizer=tokenizer)
    model, config, version, sampling_seed = load_checkpoint_model(
        model_dir=model_dir, checkpoint=checkpoint, devices=devices, max_new_tokens=max_new_tokens,
        temperature=temperature, seed=seed)
    limit = model.config.max_position_embeddings - config.max_new_tokens
    if config.max_prompt_tokens is not None:
        limit = min(limit, config.max_prompt_tokens)
    if len(record.prompt_ids) > limit:
        raise ValueError("prompt length + max_new_tokens exceeds model context or prompt limit")
    if any(t >= model.config.vocab_size for t in record.prompt_ids):
        raise ValueError("prompt token IDs must be inside the model vocabulary")
    group = generate_group(model, record, group_size=1, max_new_tokens=config.max_new_tokens,
                           temperature=config.temperature, **generation_options(model_dir, model.config, config),
                           policy_version=version, group_id=0,
                           generator=torch.Generator(device="cpu").manual_seed(sampling_seed),
                           reward_fn=lambda record, response_ids: 0.0)
    sample = group.samples[0]
    result = {"prompt_ids": record.prompt_ids, "response_ids": sample.response_ids,
              "finish_reason": sample.finish_reason, "stop_token_count": sample.stop_token_count,
              "policy_version": version, "seed": sampling_seed, "engram_device": model.engram_device}
    if tokenizer is not None:
        result.update(decoded_fields(tokenizer, sample.content_ids, "response"))
    return result


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description="Sample text or token IDs from an RL policy checkpoint")
    p.add_argument("--model-dir", required=True)
    p.add_argument("--checkpoint", required=True, help="RL step-XXXXXXXX.pt checkpoint")
    inputs = p.add_mutually_exclusive_group(required=True)
    inputs.add_argument("--prompt-ids", help="JSON list of token IDs, for example '[1,4,5]'")
    inputs.add_argument("--prompt", help="user text; uses the checkpoint chat template when available")
    inputs.add_argument("--messages", help="JSON list of role/content messages ending in a user turn")
    p.add_argument("--devices", "--device", default="cpu", help="cpu or comma-separated CUDA devices")
    p.add_argument("--max-new-tokens", type=int)
    p.add_argument("--temperature", type=float)
    p.add_argument("--seed", type=int)
    args = p.parse_args(argv)
    try:
        result = sample_checkpoint(
            model_dir=args.model_dir, checkpoint=args.checkpoint,
            prompt_ids=json.loads(args.prompt_ids) if args.prompt_ids is not None else None, prompt=args.prompt,
            messages=json.loads(args.messages) if args.messages is not None else None,
            devices=tuple(d.strip() for d in args.devices.split(",")), max_new_tokens=args.max_new_tokens,
            temperature=args.temperature, seed=args.seed)
    except (ValueError, TypeError) as exc:
        p.error(str(exc))
    print(json.dumps(result, sort_keys=True, allow_nan=False), flush=True)


if __name__ == "__main__":
    main()
