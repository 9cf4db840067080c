"""``python -m tiny_dsv41_b200.rl.sample`` (also ``python -m dsv41_train.rl.sample``): generate from
an RL checkpoint on top of its base model.

Flags and output fields follow ``dsv41_train/rl/sample.py:21-153``. The checkpoint records the
identity of the base it was trained from (config hash, weight files, text assets, random-init
flag); that identity must equal the one of the mounted model directory. The policy state is
restored into a freshly built model, and ``--seed`` seeds only the CPU sampling generator.
"""

from __future__ import annotations

import argparse
import json
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

# identity fields that tie a checkpoint to its base model
_BASE_KEYS = ("config_sha256", "random_init", "weights", "text_assets")
_SEED_LIMIT = 2 ** 63 - 1


def _read_checkpoint(path) -> dict:
    state = torch.load(path, map_location="cpu", weights_only=False)
    if not isinstance(state, dict) or state.get("format_version") not in (1, 2):
        raise ValueError("unsupported RL checkpoint format")
    if not {"config", "identity", "policy", "step"} <= state.keys():
        raise ValueError("RL checkpoint is missing config, identity, policy or step")
    identity = state["identity"]
    if not isinstance(identity, dict) or not isinstance(identity.get("random_init"), bool):
        raise ValueError("checkpoint identity must contain a boolean random_init flag")
    if not (type(state["step"]) is int and state["step"] >= 0):
        raise ValueError("checkpoint step must be a nonnegative integer")
    return state


def _check_base(identity: dict, model_dir: Path) -> None:
    mounted = run_identity(model_dir, None, identity["random_init"])
    if any(identity.get(key) != mounted.get(key) for key in _BASE_KEYS):
        raise ValueError("checkpoint base-model identity differs from the mounted model directory")


def load_checkpoint_model(*, model_dir, checkpoint, devices: Sequence[str] = ("cpu",),
                          max_new_tokens: Optional[int] = None, temperature: Optional[float] = None,
                          seed: Optional[int] = None):
    """(model in eval mode, run config, policy version, sampling seed)."""
    model_dir = Path(model_dir).resolve()
    state = _read_checkpoint(checkpoint)
    _check_base(state["identity"], model_dir)
    values = {**state["config"], "learner_devices": tuple(devices), "rollout_devices": tuple(devices),
              "rollout_engine": "native-pytorch"}
    for name, value in (("max_new_tokens", max_new_tokens), ("temperature", temperature)):
        if value is not None:
            values[name] = value
    config = RLConfig.from_dict(values)
    sampling_seed = config.seed if seed is None else seed
    if not (type(sampling_seed) is int and 0 <= sampling_seed < _SEED_LIMIT):
        raise ValueError("sampling seed must be an integer in [0, 2**63 - 1)")
    torch.set_num_threads(config.num_threads)
    model = make_model(model_dir, load_model_config(model_dir), config, devices, state["identity"]["random_init"],
                       role="actor")
    load_policy(model, state["policy"])
    model.eval()
    return model, config, state["step"], sampling_seed


def _prompt_fits(record: PromptRecord, model, config) -> None:
    room = model.config.max_position_embeddings - config.max_new_tokens
    if config.max_prompt_tokens is not None:
        room = min(room, config.max_prompt_tokens)
    if len(record.prompt_ids) > room:
        raise ValueError("prompt length + max_new_tokens exceeds model context or prompt limit")
    if max(record.prompt_ids) >= model.config.vocab_size:
        raise ValueError("prompt token IDs must be inside the model vocabulary")


def sample_checkpoint(*, model_dir, checkpoint, prompt_ids=None, prompt=None, messages=None, devices=("cpu",),
                      max_new_tokens=None, temperature=None, seed=None) -> dict:
    tokenizer = ModelTokenizer(model_dir) if (Path(model_dir) / "tokenizer.json").is_file() else None
    given = {"prompt_ids": prompt_ids, "prompt": prompt, "messages": messages}
    record = PromptRecord.from_mapping({k: v for k, v in given.items() if v is not None}, tokenizer=tokenizer)
    model, config, version, sampling_seed = load_checkpoint_model(
        model_dir=model_dir, checkpoint=checkpoint, devices=devices, max_new_tokens=max_new_tokens,
        temperature=temperature, seed=seed)
    _prompt_fits(record, model, config)
    group = generate_group(model, record, group_size=1, max_new_tokens=config.max_new_tokens,
                           temperature=config.temperature, policy_version=version, group_id=0,
                           generator=torch.Generator(device="cpu").manual_seed(sampling_seed),
                           reward_fn=lambda _record, _ids: 0.0, **generation_options(model_dir, model.config, config))
    sample = group.samples[0]
    result = {"prompt_ids": record.prompt_ids, "response_ids": sample.response_ids,
              "finish_reason": sample.finish_reason, "stop_token_count": sample.stop_token_count,
              "policy_version": version, "seed": sampling_seed, "engram_device": model.engram_device}
    if tokenizer is not None:
        result |= decoded_fields(tokenizer, sample.content_ids, "response")
    return result


def main(argv=None) -> None:
    parser = argparse.ArgumentParser(description="Generate from an RL policy checkpoint (text or token IDs)")
    parser.add_argument("--model-dir", required=True)
    parser.add_argument("--checkpoint", required=True, help="an RL step-XXXXXXXX.pt checkpoint")
    source = parser.add_mutually_exclusive_group(required=True)
    source.add_argument("--prompt-ids", help="token IDs as a JSON list, e.g. '[1,4,5]'")
    source.add_argument("--prompt", help="user text, wrapped by the checkpoint's chat template if it has one")
    source.add_argument("--messages", help="JSON list of role/content messages; the last one is the user's")
    parser.add_argument("--devices", "--device", default="cpu", help="cpu, or CUDA devices separated by commas")
    parser.add_argument("--max-new-tokens", type=int)
    parser.add_argument("--temperature", type=float)
    parser.add_argument("--seed", type=int)
    args = parser.parse_args(argv)
    as_json = lambda text: None if text is None else json.loads(text)  # noqa: E731
    try:
        result = sample_checkpoint(model_dir=args.model_dir, checkpoint=args.checkpoint,
                                   prompt_ids=as_json(args.prompt_ids), prompt=args.prompt,
                                   messages=as_json(args.messages),
                                   devices=tuple(d.strip() for d in args.devices.split(",")),
                                   max_new_tokens=args.max_new_tokens, temperature=args.temperature, seed=args.seed)
    except (ValueError, TypeError) as error:
        parser.error(str(error))
    print(json.dumps(result, sort_keys=True, allow_nan=False), flush=True)


if __name__ == "__main__":
    main()
