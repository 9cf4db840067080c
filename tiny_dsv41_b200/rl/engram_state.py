"""Engram tables shared by RL roles without copies: a sealed host baseline, private copy-on-write
views per role, and portable cumulative row deltas (``dsv41_train/rl/engram_state.py:26-326``).

* ``EngramBaseline`` writes each table once into a Linux ``memfd`` and seals it (no write,
  grow, shrink or further seals), so no process can change the baseline. Child processes
  receive duplicated file descriptors, never tensor storage. (A temp-file fallback for
  non-Linux CPU development is capped at 64 MiB.)
* ``EngramBaseline.view`` maps a table copy-on-write: a role's writes stay private pages.
* ``EngramState`` gives each role (learner / reference / actor) its tables; the learner tracks
  the rows its sparse gradients touched and exports ``{format 1, base identity,
  tables{name: {indices (sorted int64), values}}}``; loading a delta first restores every
  previously touched row from the baseline, so any cumulative snapshot can be installed.
"""

from __future__ import annotations

import fcntl
import mmap
import os
import sys
import tempfile
from copy import deepcopy
from multiprocessing.reduction import DupFd
from pathlib import Path

import torch
from torch import nn

from ..parallel.engram_offload import CPUEmbeddingLookup

_F_ADD_SEALS, _F_GET_SEALS = 1033, 1034           # Linux fcntl commands
_SEAL_SEAL, _SEAL_SHRINK, _SEAL_GROW, _SEAL_WRITE = 1, 2, 4, 8
_FALLBACK_LIMIT = 64 << 20


def create_memfd(name: str) -> int:
    if sys.platform != "linux":
        raise RuntimeError("sealed memfd requires Linux")
    return os.memfd_create(name, os.MFD_CLOEXEC | os.MFD_ALLOW_SEALING)


def memfd_seals(fd: int) -> int:
    return fcntl.fcntl(fd, getattr(fcntl, "F_GET_SEALS", _F_GET_SEALS))


def seal_memfd(fd: int) -> int:
    want = _SEAL_WRITE | _SEAL_SHRINK | _SEAL_GROW | _SEAL_SEAL
    fcntl.fcntl(fd, getattr(fcntl, "F_ADD_SEALS", _F_ADD_SEALS), want)
    got = memfd_seals(fd)
    if got & want != want:
        raise RuntimeError("Engram memfd is missing required kernel seals")
    return got


def _itemsize(dtype) -> int:
    return torch.empty((), dtype=dtype).element_size()


def validate_delta(payload, identity, shapes, dtype) -> None:
    if (not isinstance(payload, dict) or set(payload) != {"format", "base", "tables"} or payload["format"] != 1
            or type(payload["format"]) is not int or payload["base"] != identity
            or not isinstance(payload["tables"], dict) or payload["tables"].keys() != shapes.keys()):
        raise ValueError("Engram delta format or baseline identity differs")
    for name, (rows, width) in shapes.items():
        rec = payload["tables"][name]
        if not isinstance(rec, dict) or set(rec) != {"indices", "values"}:
            raise ValueError(f"invalid Engram row record: {name}")
        idx, val = rec["indices"], rec["values"]
        ok = (isinstance(idx, torch.Tensor) and idx.device.type == "cpu" and idx.dtype == torch.int64 and idx.ndim == 1
              and isinstance(val, torch.Tensor) and val.device.type == "cpu" and val.dtype == dtype
              and tuple(val.shape) == (idx.numel(), width)
              and (idx.numel() == 0 or (idx[0] >= 0 and idx[-1] < rows and not bool((idx[1:] <= idx[:-1]).any())))
              and bool(torch.isfinite(val).all()))
        if not ok:
            raise ValueError(f"invalid Engram delta indices, dtype, shape or values: {name}")


def baseline_identity(model_dir, config, dtype, random_init: bool, seed: int) -> dict:
    from .checkpoint import run_identity

    source = run_identity(model_dir, None, random_init)
    return {"source": source, "dtype": str(dtype), "seed": seed if random_init else None,
            "tables": {str(layer): [rows, config.engram_head_dim]
                       for layer, rows in zip(config.engram_layer_ids, config.engram_num_embeddings)}}


class EngramBaseline:
    chunk_rows = 131072

    def __init__(self, identity, shapes, dtype, fds) -> None:
        self.identity, self.shapes, self.dtype, self._fds = identity, shapes, dtype, fds

    @property
    def byte_size(self) -> int:
        return sum(r * w for r, w in self.shapes.values()) * _itemsize(self.dtype)

    def __getstate__(self):
        return self.identity, self.shapes, self.dtype, {n: DupFd(fd) for n, fd in self._fds.items()}

    def __setstate__(self, state):
        identity, shapes, dtype, fds = state
        self.__init__(identity, shapes, dtype, {n: d.detach() for n, d in fds.items()})

    def __del__(self):
        for fd in getattr(self, "_fds", {}).values():
            try:
                os.close(fd)
            except OSError:
                pass

    def view(self, name: str) -> torch.Tensor:
        rows, width = self.shapes[name]
        mapping = mmap.mmap(self._fds[name], rows * width * _itemsize(self.dtype), access=mmap.ACCESS_COPY)
        return torch.frombuffer(mapping, dtype=self.dtype).reshape(rows, width)

    @classmethod
    def create(cls, model_dir, config, dtype, random_init: bool, seed: int, initial_delta=None) -> "EngramBaseline":
        """Fill each table from a seeded random init, a released FP8 checkpoint or native tensors,
        then apply an optional initial delta, then seal."""
        from ..models.dsv4.checkpoint import ShardedSafeTensorReader
        from ..utils.quant import dequantize_fp8_rows
        from .checkpoint import file_sha256

        root = Path(model_dir)
        identity = baseline_identity(root, config, dtype, random_init, seed)
        shapes = {n: tuple(s) for n, s in identity["tables"].items()}
        if not shapes or dtype not in (torch.float32, torch.bfloat16):
            raise ValueError("trainable Engram requires nonempty FP32 or BF16 CPU tables")
        payload = None
        if initial_delta is not None:
            payload = torch.load(initial_delta, map_location="cpu", weights_only=True)
            validate_delta(payload, identity, shapes, dtype)
            identity = dict(identity, initial_delta_sha256=file_sha256(initial_delta))
        linux = sys.platform == "linux"
        total = sum(r * w for r, w in shapes.values()) * _itemsize(dtype)
        if not linux and total > _FALLBACK_LIMIT:
            raise RuntimeError("large Engram baselines require Linux memfd")
        reader = None if random_init else ShardedSafeTensorReader(root)
        released = reader is not None and getattr(config, "checkpoint_format", "native") == "released"
        fds: dict[str, int] = {}
        try:
            for name, (rows, width) in shapes.items():
                size = rows * width * _itemsize(dtype)
                tmp_path = None
                if linux:
                    fd = create_memfd(f"engram-{name}")
                else:
                    fd, tmp_path = tempfile.mkstemp(prefix="engram-baseline-")
                fds[name] = fd
                os.ftruncate(fd, size)
                mapping = mmap.mmap(fd, size, access=mmap.ACCESS_WRITE)
                try:
                    dst = torch.frombuffer(mapping, dtype=dtype).reshape(rows, width)
                    gen = torch.Generator().manual_seed((seed + int(name)) % (2 ** 63 - 1))
                    for start in range(0, rows, cls.chunk_rows):
                        stop = min(rows, start + cls.chunk_rows)
                        if random_init:
                            dst[start:stop].normal_(std=config.initializer_range, generator=gen)
                        elif released:
                            stem = f"layers.{name}.engram.embed"
                            dst[start:stop].copy_(dequantize_fp8_rows(reader.tensor_rows(f"{stem}.weight", start, stop),
                                                                      reader.tensor_rows(f"{stem}.scale", start, stop),
                                                                      dtype=dtype))
                        else:
                            dst[start:stop].copy_(reader.tensor_rows(f"model.engram_tables.{name}.weight", start, stop))
                    if payload is not None:
                        rec = payload["tables"][name]
                        dst.index_copy_(0, rec["indices"], rec["values"])
                    del dst
                finally:
                    mapping.close()
                    if tmp_path is not None:
                        readonly = os.open(tmp_path, os.O_RDONLY)
                        os.close(fd)
                        fds[name] = readonly
                        os.unlink(tmp_path)
                if linux:
                    seal_memfd(fd)
        except BaseException:
            for fd in fds.values():
                try:
                    os.close(fd)
                except OSError:
                    pass
            raise
        finally:
            if reader is not None:
                reader.close()
        return cls(identity, shapes, dtype, fds)


class RoleEmbedding(nn.Module):
    """A role's private view, looked up from host memory (results land on ``placement``'s device)."""

    sparse_gradients = engram_offload = True

    def __init__(self, weight: torch.Tensor, trainable: bool) -> None:
        super().__init__()
        self.weight = nn.Parameter(weight, requires_grad=trainable)
        self.register_buffer("placement", torch.empty(0, dtype=weight.dtype), persistent=False)
        self._cpu_lookup = CPUEmbeddingLookup()

    def _apply(self, fn, recurse=True):
        target = fn(self.placement)
        if target.dtype != self.weight.dtype:
            raise ValueError("Engram baseline dtype is fixed; build it in the training dtype")
        self.synchronize()
        self.placement = target
        self.clear_cache()
        return self

    def forward(self, indices):
        return self._cpu_lookup(self.weight, indices, device=self.placement.device)

    def configure_cache(self, budget: int) -> None:
        self._cpu_lookup.configure_cache(budget, self.placement.device)

    def synchronize(self) -> None:
        self._cpu_lookup.synchronize()

    def clear_cache(self) -> None:
        self._cpu_lookup.clear_cache()


class EngramState:
    def __init__(self, baseline: EngramBaseline, role: str, trainable: bool) -> None:
        if role not in {"learner", "reference", "actor"}:
            raise ValueError("unknown Engram policy role")
        self.baseline, self.role = baseline, role
        self.tables = {n: RoleEmbedding(baseline.view(n), trainable and role == "learner") for n in baseline.shapes}
        self.dirty = {n: torch.empty(0, dtype=torch.long) for n in self.tables}

    @property
    def byte_size(self) -> int:
        return self.baseline.byte_size

    def synchronize(self) -> None:
        for t in self.tables.values():
            t.synchronize()

    def mark_touched(self) -> None:
        if self.role != "learner":
            raise RuntimeError("only the learner may update Engram")
        for name, t in self.tables.items():
            g = t.weight.grad
            if g is not None:
                if not g.is_sparse:
                    raise ValueError("Engram gradients must be sparse")
                self.dirty[name] = torch.cat((self.dirty[name], g.coalesce().indices()[0])).unique(sorted=True)

    def state_dict(self) -> dict:
        self.synchronize()
        return {"format": 1, "base": deepcopy(self.baseline.identity),
                "tables": {n: {"indices": ids.clone(), "values": self.tables[n].weight.detach().index_select(0, ids)}
                           for n, ids in self.dirty.items()}}

    def validate(self, payload) -> None:
        if self.role == "reference":
            raise ValueError("the initial reference cannot load learner Engram state")
        validate_delta(payload, self.baseline.identity, self.baseline.shapes, self.baseline.dtype)

    @torch.no_grad()
    def load_state_dict(self, payload) -> None:
        self.validate(payload)
        self.synchronize()
        for name, t in self.tables.items():
            original = self.baseline.view(name)
            for ids in self.dirty[name].split(self.baseline.chunk_rows):
                t.weight.index_copy_(0, ids, original.index_select(0, ids))
            rec = payload["tables"][name]
            t.weight.index_copy_(0, rec["indices"], rec["values"])
            t.weight.grad = None
            self.dirty[name] = rec["indices"].clone()
            t.clear_cache()


__all__ = ["EngramBaseline", "EngramState", "RoleEmbedding", "baseline_identity", "create_memfd", "seal_memfd",
           "validate_delta"]
