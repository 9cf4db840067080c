"""Portable LoRA + Engram SFT bundle (``dsv41_train/sft_export.py:68-165``).

``sft-bundle-STEP/`` holds ``adapter.pt`` (the LoRA adapter, bound to the base identity),
``engram_delta.pt`` (``{format 1, base, tables{name: {indices, values}}}``: every Engram row the
SFT run touched, in global row ids, gathered from the owners' snapshot shards of the paired SFT
checkpoint) and, written last, ``manifest.json`` (``{format 1, kind "lora-engram-sft", step,
base, files{name: sha256}}``). RL consumes it through ``--initial-adapter <bundle dir>``
(``resolve_initial_bundle``), which verifies every file before use.

All ranks call ``export_sft_bundle``; rank 0 writes. Validation failures are agreed on before
the collective adapter gather, so no rank is left waiting.
"""

from __future__ import annotations

import json
import os
from dataclasses import replace
from pathlib import Path

import torch
import torch.distributed as dist

from ..lora import adapter_parameters, save_adapter
from ..rl.checkpoint import atomic_save, file_sha256
from ..rl.engram_state import baseline_identity, validate_delta


def _rank_payload(checkpoint: Path, manifest: dict, rank: int) -> dict:
    record = manifest["ranks"][rank]
    path = checkpoint / f"rank-{rank:05d}.pt"
    if file_sha256(path) != record["sha256"]:
        raise ValueError(f"incomplete or corrupt SFT owner {rank}")
    return torch.load(path, map_location="cpu", weights_only=False)


def global_rows(checkpoint, manifest: dict, base: dict) -> dict:
    """Touched rows of every owner shard, in global ids, as one validated delta."""
    checkpoint = Path(checkpoint)
    shapes = {n: tuple(s) for n, s in base["tables"].items()}
    dtype = getattr(torch, base["dtype"].removeprefix("torch."))
    names = {f"model.engram_tables.{n}.weight": n for n in shapes}
    parts = {n: [] for n in shapes}
    for rank in range(len(manifest["ranks"])):
        snapshot = _rank_payload(checkpoint, manifest, rank).get("engram_rows")
        if not isinstance(snapshot, dict) or snapshot.get("format") != 1 or snapshot["tables"].keys() != names.keys():
            raise ValueError("SFT Engram owner snapshot or table set differs")
        for full, name in names.items():
            layout, rows = snapshot["schema"][full], snapshot["tables"][full]
            start, stop = layout["row_start"], layout["row_stop"]
            total, width = shapes[name]
            if layout["global_shape"] != [total, width] or layout["dtype"] != str(dtype) or not 0 <= start <= stop <= total:
                raise ValueError("SFT Engram owner bounds, dtype or shape differ")
            validate_delta({"format": 1, "base": base, "tables": {name: rows}}, base, {name: (stop - start, width)}, dtype)
            parts[name].append((start, stop, rows))
    tables = {}
    for name, owners in parts.items():
        owners.sort(key=lambda o: (o[0], o[1]))
        end = 0
        for start, stop, _ in owners:
            if start != end:
                raise ValueError("SFT Engram owners overlap or leave missing rows")
            end = stop
        if end != shapes[name][0]:
            raise ValueError("SFT Engram owners do not cover the original table")
        tables[name] = {"indices": torch.cat([r["indices"] + s for s, _, r in owners]),
                        "values": torch.cat([r["values"] for _, _, r in owners])}
    delta = {"format": 1, "base": base, "tables": tables}
    validate_delta(delta, base, shapes, dtype)
    return delta


def _agree(error):
    if dist.is_initialized():
        status = [None] * dist.get_world_size()
        dist.all_gather_object(status, error)
        errors = [e for e in status if e]
        if errors:
            raise ValueError("SFT bundle export failed: " + "; ".join(errors))
    elif error:
        raise ValueError(error)


def export_sft_bundle(model, checkpoint, model_path, output) -> Path:
    from ..models.dsv4 import DeepSeekV41Config

    rank = dist.get_rank() if dist.is_initialized() else 0
    checkpoint, output = Path(checkpoint), Path(output)
    error, delta, base, manifest = None, None, None, None
    try:
        manager = getattr(model, "_sft_engram_checkpoint", None)
        config = DeepSeekV41Config.from_json(Path(model_path) / "config.json")
        if manager is None or not manager.tables:
            raise ValueError("bundle requires LoRA with trainable host-memory Engram rows")
        wanted = {id(p) for p in adapter_parameters(model)} | {id(t.weight) for t in manager.tables.values()}
        if {id(p) for p in model.parameters() if p.requires_grad} != wanted:
            raise ValueError("bundle cannot represent full SFT or other trainable base weights")
        dtypes = {t.weight.dtype for t in manager.tables.values()}
        if len(dtypes) != 1:
            raise ValueError("Engram bundle tables must share one dtype")
        base = baseline_identity(model_path, config, next(iter(dtypes)), False, 0)
        manifest = json.loads((checkpoint / "manifest.json").read_text())
        training = manifest["identity"].get("training_config", {})
        if training.get("mode") != "lora" or training.get("family") != "dsv4" or manifest["step"] < 1:
            raise ValueError("SFT bundle checkpoint mode, family or step differs")
        payload = _rank_payload(checkpoint, manifest, rank)
        live = manager.state_dict()["tables"]
        for name, rows in live.items():
            if any(not torch.equal(rows[k], payload["engram_rows"]["tables"][name][k]) for k in rows):
                raise ValueError("live Engram rows differ from their paired SFT checkpoint")
        if rank == 0:
            delta = global_rows(checkpoint, manifest, base)
            output.mkdir(parents=True, exist_ok=False)
    except Exception as exc:
        error = f"rank {rank}: {exc}"
    _agree(error)
    save_adapter(model, output / "adapter.pt", base_identity=base["source"])
    error = None
    try:
        if rank == 0:
            atomic_save(delta, output / "engram_delta.pt")
            bundle = {"format": 1, "kind": "lora-engram-sft", "step": manifest["step"], "base": base,
                      "files": {n: file_sha256(output / n) for n in ("adapter.pt", "engram_delta.pt")}}
            tmp = output / ".manifest.json.tmp"
            with tmp.open("x") as f:
                json.dump(bundle, f, sort_keys=True, allow_nan=False)
                f.flush()
                os.fsync(f.fileno())
            tmp.replace(output / "manifest.json")
    except Exception as exc:
        error = f"rank {rank}: {exc}"
    _agree(error)
    return output


def resolve_initial_bundle(config):
    """An ``initial_adapter`` that is a directory must be a complete, verified SFT bundle."""
    if config.initial_adapter is None or not Path(config.initial_adapter).is_dir():
        return config
    root = Path(config.initial_adapter).absolute()
    manifest = json.loads((root / "manifest.json").read_text())
    if (set(manifest) != {"format", "kind", "step", "base", "files"} or manifest["format"] != 1
            or manifest["kind"] != "lora-engram-sft" or type(manifest["step"]) is not int or manifest["step"] < 1
            or manifest["files"].keys() != {"adapter.pt", "engram_delta.pt"}
            or config.initial_engram_delta is not None or config.trainable_scope != "lora"):
        raise ValueError("invalid SFT bundle manifest, scope or conflicting explicit Engram delta")
    for name, digest in manifest["files"].items():
        if (root / name).is_symlink() or file_sha256(root / name) != digest:
            raise ValueError(f"SFT bundle file checksum differs: {name}")
    delta = torch.load(root / "engram_delta.pt", weights_only=True, map_location="cpu")
    base = manifest["base"]
    validate_delta(delta, base, {n: tuple(s) for n, s in base["tables"].items()},
                   getattr(torch, base["dtype"].removeprefix("torch.")))
    resolved = replace(config, initial_adapter=str(root / "adapter.pt"), initial_engram_delta=str(root / "engram_delta.pt"))
    resolved.validate()
    return resolved


__all__ = ["export_sft_bundle", "global_rows", "resolve_initial_bundle"]
