"""RL checkpoint and policy-artifact formats.

* ``atomic_save``: temp file + fsync + rename + directory fsync.
* Policy artifacts ``policies/policy-VVVVVVVV-<sha256>.pt`` - immutable, digest-named, staged
  then hard-linked; payload ``{version, lineage, identity, sampling, trainable, frozen, ...}``;
  activation returns a receipt ``{version, digest, lineage}`` (``validate_policy_ack``).
* Training checkpoints ``step-XXXXXXXX.pt`` (format 2): policy state, optimizer, config,
  identity, step, group cursor, rollout RNG, learner RNG, dropped groups, manager state.
* ``run_identity``: config sha256, base-weight inventory (name/size/mtime), text-asset hashes,
  data sha256 - resume refuses a different identity.
Formats follow ``dsv41_train/rl/checkpoint.py``.
"""

from __future__ import annotations

import hashlib
import json
import os
import tempfile
from pathlib import Path

import torch

FORMAT_VERSION = 2


def _sync_directory(path: Path) -> None:
    fd = os.open(path, os.O_RDONLY | getattr(os, "O_DIRECTORY", 0))
    try:
        os.fsync(fd)
    finally:
        os.close(fd)


def file_sha256(path) -> str:
    digest = hashlib.sha256()
    with Path(path).open("rb") as f:
        for chunk in iter(lambda: f.read(8 * 1024 * 1024), b""):
            digest.update(chunk)
    return digest.hexdigest()


def atomic_save(payload: dict, destination) -> None:
    destination = Path(destination)
    destination.parent.mkdir(parents=True, exist_ok=True)
    fd, temporary = tempfile.mkstemp(prefix=f".{destination.name}-", dir=destination.parent)
    try:
        with os.fdopen(fd, "wb") as f:
            torch.save(payload, f)
            f.flush()
            os.fsync(f.fileno())
        os.replace(temporary, destination)
        _sync_directory(destination.parent)
    finally:
        if os.path.exists(temporary):
            os.unlink(temporary)


def run_identity(model_dir, data_path, random_init: bool, *, eval_data_path=None) -> dict:
    model_dir = Path(model_dir)
    config = model_dir / "config.json"
    identity = {"config_sha256": file_sha256(config) if config.exists() else None, "random_init": bool(random_init)}
    weights = sorted(model_dir.glob("*.safetensors")) + sorted(model_dir.glob("*.index.json"))
    identity["weights"] = [{"name": p.name, "bytes": p.stat().st_size, "mtime_ns": p.stat().st_mtime_ns}
                           for p in weights] if not random_init else []
    identity["text_assets"] = {p.name: file_sha256(p) for p in sorted(model_dir.glob("tokenizer*.json"))
                               + sorted(model_dir.glob("*.jinja")) if p.is_file()}
    if data_path is not None:
        identity["data_sha256"] = file_sha256(data_path)
    if eval_data_path is not None:
        identity["eval_data_sha256"] = file_sha256(eval_data_path)
    return identity


def validate_identity(saved: dict, current: dict) -> None:
    if json.dumps(saved, sort_keys=True) != json.dumps(current, sort_keys=True):
        raise ValueError("checkpoint run identity differs from the current run")


def policy_state(model) -> dict:
    return {"trainable": model.trainable_state_dict(), "frozen": model.frozen_state_dict()}


def load_policy(model, state: dict) -> None:
    model.load_trainable_state_dict(state["trainable"])
    model.load_frozen_state_dict(state["frozen"])


def publish_policy_artifact(model, version: int, directory, *, lineage: str, identity: dict, sampling: dict) -> dict:
    if type(version) is not int or version < 0 or not isinstance(lineage, str) or not lineage:
        raise ValueError("policy artifact requires a nonnegative version and run lineage")
    directory = Path(directory).resolve()
    directory.mkdir(parents=True, exist_ok=True)
    payload = {"version": version, "lineage": lineage, "identity": identity, "sampling": sampling, **policy_state(model)}
    with tempfile.TemporaryDirectory(prefix=".policy-stage-", dir=directory) as tmp:
        staged = Path(tmp) / "payload.pt"
        atomic_save(payload, staged)
        digest = file_sha256(staged)
        destination = directory / f"policy-{version:08d}-{digest}.pt"
        try:
            os.link(staged, destination)
        except FileExistsError:
            if file_sha256(destination) != digest:
                raise ValueError("existing policy artifact digest mismatch") from None
        _sync_directory(directory)
    return {"version": version, "digest": digest, "path": str(destination), "lineage": lineage,
            "identity": identity, "sampling": sampling}


def load_policy_artifact(model, artifact: dict) -> dict:
    digest = artifact.get("digest")
    if not isinstance(digest, str) or len(digest) != 64 or file_sha256(artifact["path"]) != digest:
        raise ValueError("policy artifact digest mismatch")
    snapshot = torch.load(artifact["path"], map_location="cpu", weights_only=True)
    for key in ("version", "lineage", "identity", "sampling"):
        if snapshot.get(key) != artifact.get(key):
            raise ValueError(f"policy artifact metadata mismatch: {key}")
    load_policy(model, snapshot)
    return {"version": artifact["version"], "digest": digest, "lineage": artifact["lineage"]}


def validate_policy_ack(ack: dict, artifact: dict) -> None:
    expected = {"version": artifact["version"], "digest": artifact["digest"], "lineage": artifact["lineage"]}
    if {k: ack.get(k) for k in expected} != expected:
        raise RuntimeError(f"rollout activation acknowledged {ack!r}, expected {expected!r}")


def save_training_checkpoint(path, model, optimizer, *, step: int, config, identity: dict, next_group_id: int,
                             rollout_rng_state, dropped_groups: int, manager_state=None,
                             policy_publication=None) -> None:
    payload = {"format_version": FORMAT_VERSION, "step": step, "policy": policy_state(model),
               "optimizer": optimizer.state_dict(), "config": config.to_dict(), "identity": identity,
               "next_group_id": next_group_id, "rollout_rng_state": rollout_rng_state,
               "learner_rng_state": torch.get_rng_state(), "dropped_groups": dropped_groups,
               "manager_state": manager_state, "policy_publication": policy_publication}
    if torch.cuda.is_available():
        payload["cuda_rng_state"] = [s for s in torch.cuda.get_rng_state_all()]
    atomic_save(payload, path)


def load_training_checkpoint(path, model, optimizer, config, identity: dict) -> dict:
    state = torch.load(path, map_location="cpu", weights_only=False)
    if state.get("format_version") not in (1, FORMAT_VERSION):
        raise ValueError("unsupported RL checkpoint format")
    validate_identity(state["identity"], identity)
    saved = dict(state["config"])
    current = config.to_dict()
    for key in ("group_size", "max_new_tokens", "temperature", "reward", "trainable_scope"):
        if json.dumps(saved.get(key)) != json.dumps(current.get(key)):
            raise ValueError(f"checkpoint config differs for {key}")
    load_policy(model, state["policy"])
    optimizer.load_state_dict(state["optimizer"])
    torch.set_rng_state(state["learner_rng_state"])
    return state


__all__ = ["atomic_save", "file_sha256", "load_policy", "load_policy_artifact", "load_training_checkpoint",
           "policy_state", "publish_policy_artifact", "run_identity", "save_training_checkpoint",
           "validate_identity", "validate_policy_ack"]
