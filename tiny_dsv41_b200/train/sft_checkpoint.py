"""Same-topology SFT snapshots (``dsv41_train/sft_checkpoint.py`` semantics).

A snapshot directory holds ``manifest.json`` (format, step, data position, world size, run
identity, per-rank schema digest) and one ``rank-XXXXX.pt`` per rank with that rank's local
shards of every trainable parameter and persistent buffer (Engram tables excluded), plus its
optimizer state. Frozen parameters are not saved: they reload from the identified base model.
Loading requires the same world size, topology (tensor names, global/local shapes, dtypes,
placements, expert / row ownership) and identity; nothing is resharded.

Writes are atomic per file; the manifest is written last by rank 0 after every rank finished,
so a directory without a manifest is an incomplete snapshot and is refused.
"""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

import torch
import torch.distributed as dist

from ..rl.checkpoint import atomic_save, file_sha256

FORMAT = 1


def _position():
    return (dist.get_rank(), dist.get_world_size()) if dist.is_initialized() else (0, 1)


def _local(t):
    return t.to_local() if hasattr(t, "to_local") else t


def _layout(t) -> dict:
    out = {"shape": list(t.shape), "local_shape": list(_local(t).shape), "dtype": str(t.dtype)}
    if hasattr(t, "placements"):
        out["placements"] = [str(p) for p in t.placements]
        out["mesh"] = t.device_mesh.mesh.tolist()
    return out


def _tensors(model):
    manager = getattr(model, "_sft_engram_checkpoint", None)
    rows = manager.parameter_names if manager is not None else frozenset()
    params = {n: p for n, p in model.named_parameters() if p.requires_grad and n not in rows}
    buffers = {}
    for prefix, module in model.named_modules():
        for name, value in module.named_buffers(recurse=False):
            full = f"{prefix}.{name}" if prefix else name
            if name not in module._non_persistent_buffers_set and ".engram_tables." not in f".{full}":
                buffers[full] = value
    return params, buffers


def _ownership(model) -> dict:
    fields = ("layer_id", "expert_start", "num_experts", "row_start", "row_stop")
    return {n: {f: int(getattr(m, f)) for f in fields if isinstance(getattr(m, f, None), int)}
            for n, m in model.named_modules() if any(isinstance(getattr(m, f, None), int) for f in fields)}


def _schema(model, optimizer) -> dict:
    params, buffers = _tensors(model)
    names = {id(p): n for n, p in params.items()}
    manager = getattr(model, "_sft_engram_checkpoint", None)
    if manager is not None:  # row-snapshot tables are optimizer members without saved state
        names.update({id(t.weight): n for n, t in manager.tables.items()})
    groups = []
    for group in optimizer.param_groups:
        if any(id(p) not in names for p in group["params"]):
            raise ValueError("optimizer must contain only trainable model parameters")
        groups.append({"params": [names[id(p)] for p in group["params"]],
                       **{k: v for k, v in group.items() if k != "params" and isinstance(v, (int, float, bool, str))}})
    schema = {"parameters": {n: _layout(p) for n, p in params.items()},
              "buffers": {n: _layout(b) for n, b in buffers.items()}, "ownership": _ownership(model),
              "optimizer": {"type": type(optimizer).__name__, "groups": groups}}
    if manager is not None:
        schema["engram_rows"] = manager.schema
    return schema


def _digest(value) -> str:
    return hashlib.sha256(json.dumps(value, sort_keys=True).encode()).hexdigest()


def _gather(value):
    _, world = _position()
    out = [None] * world
    if dist.is_initialized():
        dist.all_gather_object(out, value)
    else:
        out[0] = value
    return out


def _optimizer_state(optimizer, params) -> dict:
    names = {id(p): n for n, p in params.items()}
    state = {}
    for p, fields in optimizer.state.items():
        if id(p) not in names:  # Engram row tables: plain SGD keeps no state
            continue
        state[names[id(p)]] = {k: (_local(v).detach().cpu().clone() if isinstance(v, torch.Tensor) else v)
                               for k, v in fields.items()}
    return state


def save_checkpoint(directory, model, optimizer, *, step: int, identity: dict, data_position: int) -> Path:
    directory = Path(directory)
    rank, world = _position()
    if rank == 0:
        directory.mkdir(parents=True, exist_ok=True)
        manifest = directory / "manifest.json"
        if manifest.exists():
            manifest.unlink()
    if dist.is_initialized():
        dist.barrier()
    schema = _schema(model, optimizer)
    params, buffers = _tensors(model)
    payload = {"format": FORMAT, "rank": rank, "world_size": world, "step": step, "schema": schema,
               "parameters": {n: _local(p).detach().cpu().clone() for n, p in params.items()},
               "buffers": {n: _local(b).detach().cpu().clone() for n, b in buffers.items()},
               "optimizer": _optimizer_state(optimizer, params)}
    manager = getattr(model, "_sft_engram_checkpoint", None)
    if manager is not None:
        payload["engram_rows"] = manager.state_dict()
    path = directory / f"rank-{rank:05d}.pt"
    atomic_save(payload, path)
    records = _gather({"rank": rank, "sha256": file_sha256(path), "schema": _digest(schema)})
    if rank == 0:
        manifest = {"format": FORMAT, "step": step, "data_position": data_position, "world_size": world,
                    "identity": identity, "ranks": records}
        tmp = directory / ".manifest.json.tmp"
        tmp.write_text(json.dumps(manifest, indent=2, sort_keys=True) + "\n", encoding="utf-8")
        tmp.replace(directory / "manifest.json")
    if dist.is_initialized():
        dist.barrier()
    return directory


def _restore_like(param, value):
    """Optimizer tensors take the parameter's device and, for sharded parameters, its placement."""
    if not isinstance(value, torch.Tensor) or value.ndim == 0:
        return value
    local = value.to(_local(param).device)
    if hasattr(param, "device_mesh"):
        from torch.distributed.tensor import DTensor

        return DTensor.from_local(local, param.device_mesh, param.placements, run_check=False, shape=param.shape,
                                  stride=param.stride())
    return local


@torch.no_grad()
def load_checkpoint(directory, model, optimizer, *, identity: dict) -> tuple[int, int]:
    """Restore this rank's shards and optimizer state; returns (step, data_position)."""
    directory = Path(directory)
    rank, world = _position()
    manifest_path = directory / "manifest.json"
    if not manifest_path.is_file():
        raise FileNotFoundError(f"incomplete SFT checkpoint (no manifest): {directory}")
    manifest = json.loads(manifest_path.read_text(encoding="utf-8"))
    if manifest.get("format") != FORMAT or manifest.get("world_size") != world:
        raise ValueError("SFT checkpoint format or world size differs (this format does not reshard)")
    if json.dumps(manifest["identity"], sort_keys=True) != json.dumps(identity, sort_keys=True):
        raise ValueError("SFT checkpoint run identity differs from the current run")
    record = manifest["ranks"][rank]
    path = directory / f"rank-{rank:05d}.pt"
    if record["rank"] != rank or file_sha256(path) != record["sha256"]:
        raise ValueError(f"SFT checkpoint shard digest mismatch: {path}")
    payload = torch.load(path, map_location="cpu", weights_only=False)
    schema = _schema(model, optimizer)
    if _digest(schema) != record["schema"] or _digest(payload["schema"]) != record["schema"]:
        raise ValueError("SFT checkpoint topology differs from the current model and optimizer")
    params, buffers = _tensors(model)
    manager = getattr(model, "_sft_engram_checkpoint", None)
    if manager is not None:
        manager.validate(payload.get("engram_rows"))
    for n, p in params.items():
        _local(p).copy_(payload["parameters"][n])
    for n, b in buffers.items():
        _local(b).copy_(payload["buffers"][n])
    state = {}
    for n, fields in payload["optimizer"].items():
        p = params[n]
        state[p] = {k: _restore_like(p, v) for k, v in fields.items()}
    optimizer.state.clear()
    optimizer.state.update(state)
    if manager is not None:
        manager.load_state_dict(payload["engram_rows"])
    gathered = _gather(manifest["step"])
    if len(set(gathered)) != 1:
        raise ValueError("ranks restored different steps")
    return int(manifest["step"]), int(manifest["data_position"])


__all__ = ["load_checkpoint", "save_checkpoint"]
