"""Rank-local snapshots of trainable host-memory Engram rows (``dsv41_train/sft_engram.py:30-183``).

Only the rows SGD touched since the base was loaded are saved (cumulative, sorted int64 local
row ids + their values); the base table itself is never copied. Restoring a snapshot first
re-reads, from the mounted released checkpoint (FP8 E4M3 rows with per-32 E8M0 scales), every
row that is dirty now but absent from the snapshot, then writes the snapshot's rows. Snapshot
format: ``{"format": 1, "schema": {name: {global_shape, local_shape, row_start, row_stop, dtype}},
"tables": {name: {"indices", "values"}}}``.
"""

from __future__ import annotations

import re
from copy import deepcopy

import torch

from ..utils.quant import dequantize_fp8_rows
from ..utils.safetensors_io import ShardedSafeTensorReader


def trainable_engram_tables(model) -> dict:
    return {(f"{n}.weight" if n else "weight"): m for n, m in model.named_modules()
            if getattr(m, "engram_offload", False) and getattr(m, "sparse_gradients", False)
            and m.weight.requires_grad}


def _chunk_rows(width: int) -> int:
    return max(1, (4 << 20) // (24 * width))  # bounds decode temporaries to ~4 MiB


class ReleasedEngramRows:
    """Global rows of a released checkpoint's Engram tables, read and dequantised on demand."""

    def __init__(self, model_path, schema: dict) -> None:
        self.model_path, self.schema = model_path, deepcopy(schema)
        self.sources = {}
        for name in schema:
            m = re.search(r"(?:^|\.)engram_tables\.(\d+)\.weight$", name)
            if m is None:
                raise ValueError(f"cannot identify released Engram layer: {name}")
            self.sources[name] = f"layers.{m[1]}.engram.embed"

    def __call__(self, name: str, global_ids: torch.Tensor) -> torch.Tensor:
        rows, width = self.schema[name]["global_shape"]
        dtype = getattr(torch, self.schema[name]["dtype"].removeprefix("torch."))
        if global_ids.numel() > _chunk_rows(width):
            raise ValueError("Engram base read exceeds the bounded row chunk")
        out = torch.empty((global_ids.numel(), width), dtype=dtype)
        if not global_ids.numel():
            return out
        stem = self.sources[name]
        with ShardedSafeTensorReader(self.model_path) as reader:
            for suffix, shape, storage in (("weight", [rows, width], "F8_E4M3"), ("scale", [rows, width // 32], "F8_E8M0")):
                meta = reader.metadata(f"{stem}.{suffix}")
                if width % 32 or meta["shape"] != shape or meta["dtype"] != storage:
                    raise ValueError(f"invalid released Engram layout for {stem}.{suffix}")
            # read maximal runs of consecutive ids only
            cuts = [0, *((global_ids[1:] != global_ids[:-1] + 1).nonzero().flatten() + 1).tolist(), global_ids.numel()]
            for a, b in zip(cuts, cuts[1:]):
                start, stop = int(global_ids[a]), int(global_ids[b - 1]) + 1
                out[a:b].copy_(dequantize_fp8_rows(reader.tensor_rows(f"{stem}.weight", start, stop),
                                                   reader.tensor_rows(f"{stem}.scale", start, stop), dtype=dtype))
        return out


class EngramRowCheckpoint:
    def __init__(self, model, optimizer, read_base_rows) -> None:
        self.tables = trainable_engram_tables(model)
        self.parameter_names = frozenset(self.tables)
        self.read_base_rows = read_base_rows
        self._schema = {}
        for name, t in self.tables.items():
            w = t.weight
            if (hasattr(w, "device_mesh") or w.device.type != "cpu" or w.dtype not in (torch.float32, torch.bfloat16)
                    or w.ndim != 2 or not 0 <= t.row_start <= t.row_stop <= t.global_num_embeddings
                    or tuple(w.shape) != (t.row_stop - t.row_start, t.embedding_dim)):
                raise ValueError(f"invalid CPU Engram owner layout: {name}")
            self._schema[name] = {"global_shape": [t.global_num_embeddings, t.embedding_dim],
                                  "local_shape": list(w.shape), "row_start": t.row_start, "row_stop": t.row_stop,
                                  "dtype": str(w.dtype)}
        self.dirty = {n: torch.empty(0, dtype=torch.long) for n in self.tables}
        if type(optimizer) is not torch.optim.SGD:
            raise ValueError("sparse Engram checkpoints require native SGD")
        groups = {id(p): g for g in optimizer.param_groups for p in g["params"]}
        for t in self.tables.values():
            g = groups.get(id(t.weight))
            if g is None or any(g.get(k) for k in ("momentum", "weight_decay", "maximize", "differentiable", "foreach",
                                                   "fused")):
                raise ValueError("Engram checkpoint tracking requires owned plain sparse SGD parameters")
        self.handle = optimizer.register_step_post_hook(self._after_step)

    @property
    def schema(self) -> dict:
        return deepcopy(self._schema)

    def remove(self) -> None:
        self.handle.remove()

    def _after_step(self, _opt, _args, _kwargs) -> None:
        for name, t in self.tables.items():
            g = t.weight.grad
            if g is not None:
                if not g.is_sparse:
                    raise ValueError("Engram checkpoint tracking requires sparse gradients")
                self.dirty[name] = torch.cat((self.dirty[name], g.coalesce().indices()[0])).unique(sorted=True)

    def _drain(self) -> None:
        for t in self.tables.values():
            t.synchronize()

    def state_dict(self) -> dict:
        self._drain()
        return {"format": 1, "schema": self.schema,
                "tables": {n: {"indices": ids.clone(), "values": self.tables[n].weight.detach().index_select(0, ids)}
                           for n, ids in self.dirty.items()}}

    def validate(self, payload) -> None:
        if (not isinstance(payload, dict) or set(payload) != {"format", "schema", "tables"} or payload["format"] != 1
                or payload["schema"] != self._schema or not isinstance(payload["tables"], dict)
                or payload["tables"].keys() != self.tables.keys()):
            raise ValueError("Engram row snapshot schema or parameter names differ")
        for name, t in self.tables.items():
            rec = payload["tables"][name]
            if not isinstance(rec, dict) or set(rec) != {"indices", "values"}:
                raise ValueError(f"invalid Engram row record: {name}")
            idx, val = rec["indices"], rec["values"]
            ok = (isinstance(idx, torch.Tensor) and idx.device.type == "cpu" and idx.dtype == torch.int64
                  and idx.ndim == 1 and isinstance(val, torch.Tensor) and val.device.type == "cpu"
                  and val.dtype == t.weight.dtype and tuple(val.shape) == (idx.numel(), t.embedding_dim)
                  and (idx.numel() == 0 or (idx[0] >= 0 and idx[-1] < t.weight.shape[0]
                                            and not bool((idx[1:] <= idx[:-1]).any())))
                  and bool(torch.isfinite(val).all()))
            if not ok:
                raise ValueError(f"invalid Engram row indices, shape, dtype or values: {name}")

    @torch.no_grad()
    def load_state_dict(self, payload) -> None:
        self.validate(payload)
        self._drain()
        for name, t in self.tables.items():
            rec, old = payload["tables"][name], self.dirty[name]
            incoming = rec["indices"]
            pos = torch.searchsorted(incoming, old)
            keep = pos < incoming.numel()
            if incoming.numel():
                keep &= incoming[pos.clamp_max(incoming.numel() - 1)] == old
            for ids in old[~keep].split(_chunk_rows(t.embedding_dim)):
                if not ids.numel():
                    continue
                values = self.read_base_rows(name, ids + t.row_start)
                if (not isinstance(values, torch.Tensor) or values.dtype != t.weight.dtype
                        or tuple(values.shape) != (ids.numel(), t.embedding_dim) or not bool(torch.isfinite(values).all())):
                    raise ValueError(f"invalid original Engram rows returned for {name}")
                t.weight.index_copy_(0, ids, values)
            t.weight.index_copy_(0, incoming, rec["values"])
            t.weight.grad = None
            self.dirty[name] = incoming.clone()
            t.clear_cache()


def build_engram_checkpoint(model, model_path, optimizer):
    """After the base is loaded and the sparse SGD hooks are installed."""
    if not trainable_engram_tables(model):
        return None
    manager = EngramRowCheckpoint(model, optimizer, None)
    try:
        manager.read_base_rows = ReleasedEngramRows(model_path, manager.schema)
    except Exception:
        manager.remove()
        raise
    return manager


__all__ = ["EngramRowCheckpoint", "ReleasedEngramRows", "build_engram_checkpoint", "trainable_engram_tables"]
