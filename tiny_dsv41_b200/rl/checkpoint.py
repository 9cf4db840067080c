"""RL checkpoint and policy-artifact files.

Formats are the ones of ``dsv41_train/rl/checkpoint.py`` (a run resumes, samples and evaluates
from either side's files):

* Policy artifacts ``policies/policy-VVVVVVVV-<sha256>.pt``: immutable and named by the sha256
  of their bytes; payload ``{version, lineage, identity, sampling, trainable, frozen}``. Publishing
  writes the payload to a staging file in the same directory and hard-links it under its digest
  name, so a reader sees either no file or the complete one. The sampler acknowledges an
  activation with ``{version, digest, lineage}``.
* Training checkpoints ``step-XXXXXXXX.pt`` (format 2; format 1 still loads): the policy state,
  optimizer, run config and identity, step, group cursor, sampler and learner RNG states, dropped
  group count, manager recovery state and the last published policy.
* Run identity: sha256 of config.json, the base-weight inventory (name, size, mtime; empty for a
  random init), sha256 of the tokenizer / chat-template files and of the data files. Resuming
  under a different identity is refused.

Every file is written to a temporary name, fsynced, renamed into place and its directory fsynced.
"""

from __future__ import annotations

import hashlib
import json
import os
import tempfile
from pathlib import Path

import torch

FORMAT_VERSION = 2
_HASH_CHUNK = 8 << 20
# run-config fields a resumed run may not change
_RESUME_INVARIANT = ("group_size", "max_new_tokens", "temperature", "reward", "trainable_scope")
_ACK_FIELDS = ("version", "digest", "lineage")


def _fsync_directory(directory: Path) -> None:
    handle = os.open(directory, os.O_RDONLY | getattr(os, "O_DIRECTORY", 0))
    try:
        os.fsync(handle)
    finally:
        os.close(handle)


def file_sha256(path) -> str:
    hasher = hashlib.sha256()
    with open(path, "rb") as source:
        while block := source.read(_HASH_CHUNK):
            hasher.update(block)
    return hasher.hexdigest()


def atomic_save(payload: dict, destination) -> None:
    target = Path(destination)
    target.parent.mkdir(parents=True, exist_ok=True)
    handle, scratch = tempfile.mkstemp(prefix=f".{target.name}-", dir=target.parent)
    try:
        with os.fdopen(handle, "wb") as sink:
            torch.save(payload, sink)
            sink.flush()
            os.fsync(sink.fileno())
        os.replace(scratch, target)
        _fsync_directory(target.parent)
    finally:
        if os.path.exists(scratch):
            os.unlink(scratch)


# -- run identity -----------------------------------------------------------------------------------
def _weight_inventory(model_dir: Path) -> list[dict]:
    files = [*sorted(model_dir.glob("*.safetensors")), *sorted(model_dir.glob("*.index.json"))]
    inventory = []
    for path in files:
        info = path.stat()
        inventory.append({"name": path.name, "bytes": info.st_size, "mtime_ns": info.st_mtime_ns})
    return inventory


def _text_asset_hashes(model_dir: Path) -> dict:
    assets = [*sorted(model_dir.glob("tokenizer*.json")), *sorted(model_dir.glob("*.jinja"))]
    return {path.name: file_sha256(path) for path in assets if path.is_file()}


def run_identity(model_dir, data_path, random_init: bool, *, eval_data_path=None) -> dict:
    model_dir = Path(model_dir)
    config = model_dir / "config.json"
    identity = {
        "config_sha256": file_sha256(config) if config.exists() else None,
        "random_init": bool(random_init),
        "weights": [] if random_init else _weight_inventory(model_dir),
        "text_assets": _text_asset_hashes(model_dir),
    }
    for key, path in (("data_sha256", data_path), ("eval_data_sha256", eval_data_path)):
        if path is not None:
            identity[key] = file_sha256(path)
    return identity


def _canonical(value) -> str:
    return json.dumps(value, sort_keys=True)


def validate_identity(saved: dict, current: dict) -> None:
    if _canonical(saved) != _canonical(current):
        raise ValueError("checkpoint run identity differs from the current run")


# -- policy state and artifacts ---------------------------------------------------------------------
def policy_state(model) -> dict:
    return {"trainable": model.trainable_state_dict(), "frozen": model.frozen_state_dict()}


def load_policy(model, state: dict) -> None:
    model.load_trainable_state_dict(state["trainable"])
    model.load_frozen_state_dict(state["frozen"])


def publish_policy_artifact(model, version: int, directory, *, lineage: str, identity: dict, sampling: dict) -> dict:
    if not (type(version) is int and version >= 0 and isinstance(lineage, str) and lineage):
        raise ValueError("policy artifact requires a nonnegative version and run lineage")
    directory = Path(directory).resolve()
    directory.mkdir(parents=True, exist_ok=True)
    metadata = {"version": version, "lineage": lineage, "identity": identity, "sampling": sampling}
    with tempfile.TemporaryDirectory(prefix=".policy-stage-", dir=directory) as stage:
        staged = Path(stage) / "payload.pt"
        atomic_save({**metadata, **policy_state(model)}, staged)
        digest = file_sha256(staged)
        final = directory / f"policy-{version:08d}-{digest}.pt"
        try:
            os.link(staged, final)
        except FileExistsError:  # same name means the same bytes, unless the file was altered
            if file_sha256(final) != digest:
                raise ValueError("existing policy artifact digest mismatch") from None
        _fsync_directory(directory)
    return {"version": version, "digest": digest, "path": str(final), "lineage": lineage, "identity": identity,
            "sampling": sampling}


def load_policy_artifact(model, artifact: dict) -> dict:
    digest = artifact.get("digest")
    if not (isinstance(digest, str) and len(digest) == 64) or file_sha256(artifact["path"]) != digest:
        raise ValueError("policy artifact digest mismatch")
    payload = torch.load(artifact["path"], map_location="cpu", weights_only=True)
    for key in ("version", "lineage", "identity", "sampling"):
        if payload.get(key) != artifact.get(key):
            raise ValueError(f"policy artifact metadata mismatch: {key}")
    load_policy(model, payload)
    return {key: artifact[key] if key != "digest" else digest for key in _ACK_FIELDS}


def validate_policy_ack(ack: dict, artifact: dict) -> None:
    expected = {key: artifact[key] for key in _ACK_FIELDS}
    if any(ack.get(key) != value for key, value in expected.items()):
        raise RuntimeError(f"rollout activation acknowledged {ack!r}, expected {expected!r}")


# -- training checkpoints ---------------------------------------------------------------------------
def save_training_checkpoint(path, model, optimizer, *, step: int, config, identity: dict, next_group_id: int,
                             rollout_rng_state, dropped_groups: int, manager_state=None,
                             policy_publication=None) -> None:
    payload = {
        "format_version": FORMAT_VERSION, "step": step, "policy": policy_state(model),
        "optimizer": optimizer.state_dict(), "config": config.to_dict(), "identity": identity,
        "next_group_id": next_group_id, "rollout_rng_state": rollout_rng_state,
        "learner_rng_state": torch.get_rng_state(), "dropped_groups": dropped_groups,
        "manager_state": manager_state, "policy_publication": policy_publication,
    }
    if torch.cuda.is_available():
        payload["cuda_rng_state"] = list(torch.cuda.get_rng_state_all())
    atomic_save(payload, path)


def load_training_checkpoint(path, model, optimizer, config, identity: dict) -> dict:
    state = torch.load(path, map_location="cpu", weights_only=False)
    if state.get("format_version") not in (1, FORMAT_VERSION):
        raise ValueError("unsupported RL checkpoint format")
    validate_identity(state["identity"], identity)
    saved, current = state["config"], config.to_dict()
    for key in _RESUME_INVARIANT:
        if _canonical(saved.get(key)) != _canonical(current.get(key)):
            raise ValueError(f"checkpoint config differs for {key}")
    load_policy(model, state["policy"])
    optimizer.load_state_dict(state["optimizer"])
    torch.set_rng_state(state["learner_rng_state"])
    return state


__all__ = ["FORMAT_VERSION", "atomic_save", "file_sha256", "load_policy", "load_policy_artifact",
           "load_training_checkpoint", "policy_state", "publish_policy_artifact", "run_identity",
           "save_training_checkpoint", "validate_identity", "validate_policy_ack"]
