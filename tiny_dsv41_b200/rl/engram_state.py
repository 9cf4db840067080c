"""Engram tables shared by the RL roles without copies: one sealed host baseline, a private
copy-on-write view per role, and portable cumulative row deltas.

Behaviour of ``dsv41_train/rl/engram_state.py:26-326`` (the delta file is read by the rollout
service and by SFT export):

* The baseline holds each table once, in a Linux ``memfd`` that is filled and then sealed against
  writes, growth, shrinking and further seals, so no process can change it afterwards. Other
  processes receive duplicated file descriptors, never tensor storage. Off Linux (CPU
  development only) a deleted temporary file stands in, up to 64 MiB.
* Each role (learner / reference / actor) maps every table copy-on-write: its writes stay in its
  own pages.
* The learner records the rows its sparse gradients touched and exports
  ``{"format": 1, "base": identity, "tables": {name: {"indices": sorted int64, "values"}}}``.
  Installing a delta first restores every row the role had touched from the baseline, so any
  cumulative snapshot can be loaded in any order.
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

# Linux fcntl commands and seal bits (older Python builds lack the names)
_F_ADD_SEALS = getattr(fcntl, "F_ADD_SEALS", 1033)
_F_GET_SEALS = getattr(fcntl, "F_GET_SEALS", 1034)
_SEAL_SEAL, _SEAL_SHRINK, _SEAL_GROW, _SEAL_WRITE = 1, 2, 4, 8
_ALL_SEALS = _SEAL_WRITE | _SEAL_SHRINK | _SEAL_GROW | _SEAL_SEAL
_FALLBACK_LIMIT = 64 << 20
ROLES = ("learner", "reference", "actor")


def create_memfd(name: str) -> int:
    if sys.platform != "linux":
        raise RuntimeError("sealed memfd requires Linux")
    return os.memfd_create(name, os.MFD_CLOEXEC | os.MFD_ALLOW_SEALING)


def memfd_seals(fd: int) -> int:
    return fcntl.fcntl(fd, _F_GET_SEALS)


def seal_memfd(fd: int) -> int:
    fcntl.fcntl(fd, _F_ADD_SEALS, _ALL_SEALS)
    present = memfd_seals(fd)
    if present & _ALL_SEALS != _ALL_SEALS:
        raise RuntimeError("Engram memfd is missing required kernel seals")
    return present


def _bytes_per_value(dtype) -> int:
    return torch.empty((), dtype=dtype).element_size()


def _delta_table_ok(record, rows: int, width: int, dtype) -> bool:
    if not (isinstance(record, dict) and set(record) == {"indices", "values"}):
        return False
    ids, values = record["indices"], record["values"]
    if not (isinstance(ids, torch.Tensor) and ids.device.type == "cpu" and ids.dtype == torch.int64 and ids.ndim == 1):
        return False
    if not (isinstance(values, torch.Tensor) and values.device.type == "cpu" and values.dtype == dtype
            and tuple(values.shape) == (ids.numel(), width)):
        return False
    if ids.numel() and not (int(ids[0]) >= 0 and int(ids[-1]) < rows and bool((ids[1:] > ids[:-1]).all())):
        return False  # indices must be strictly increasing and inside the table
    return bool(torch.isfinite(values).all())


def validate_delta(payload, identity, shapes, dtype) -> None:
    header_ok = (isinstance(payload, dict) and set(payload) == {"format", "base", "tables"}
                 and type(payload["format"]) is int and payload["format"] == 1 and payload["base"] == identity
                 and isinstance(payload["tables"], dict) and payload["tables"].keys() == shapes.keys())
    if not header_ok:
        raise ValueError("Engram delta format or baseline identity differs")
    for name, (rows, width) in shapes.items():
        record = payload["tables"][name]
        if not (isinstance(record, dict) and set(record) == {"indices", "values"}):
            raise ValueError(f"invalid Engram row record: {name}")
        if not _delta_table_ok(record, rows, width, dtype):
            raise ValueError(f"invalid Engram delta indices, dtype, shape or values: {name}")


def baseline_identity(model_dir, config, dtype, random_init: bool, seed: int) -> dict:
    from .checkpoint import run_identity

    tables = {str(layer): [rows, config.engram_head_dim]
              for layer, rows in zip(config.engram_layer_ids, config.engram_num_embeddings)}
    return {"source": run_identity(model_dir, None, random_init), "dtype": str(dtype),
            "seed": seed if random_init else None, "tables": tables}


class _TableSource:
    """Produces the initial rows of one table in chunks: seeded random init, released FP8 rows,
    or native tensors of the checkpoint."""

    def __init__(self, reader, config, released: bool, random_init: bool, seed: int) -> None:
        self.reader, self.config, self.released, self.random_init, self.seed = reader, config, released, random_init, seed

    def fill(self, name: str, table: torch.Tensor, chunk: int) -> None:
        from ..utils.quant import dequantize_fp8_rows

        generator = torch.Generator().manual_seed((self.seed + int(name)) % (2 ** 63 - 1))
        for start in range(0, table.shape[0], chunk):
            stop = min(table.shape[0], start + chunk)
            rows = table[start:stop]
            if self.random_init:
                rows.normal_(std=self.config.initializer_range, generator=generator)
            elif self.released:
                stem = f"layers.{name}.engram.embed"
                rows.copy_(dequantize_fp8_rows(self.reader.tensor_rows(f"{stem}.weight", start, stop),
                                               self.reader.tensor_rows(f"{stem}.scale", start, stop),
                                               dtype=table.dtype))
            else:
                rows.copy_(self.reader.tensor_rows(f"model.engram_tables.{name}.weight", start, stop))


def _new_table_file(name: str, size: int, sealed: bool) -> tuple[int, str | None]:
    if sealed:
        fd, path = create_memfd(f"engram-{name}"), None
    else:
        fd, path = tempfile.mkstemp(prefix="engram-baseline-")
    os.ftruncate(fd, size)
    return fd, path


def _freeze_fallback(fd: int, path: str) -> int:
    """Without memfd seals: keep only a read-only descriptor of the (deleted) temporary file."""
    readonly = os.open(path, os.O_RDONLY)
    os.close(fd)
    os.unlink(path)
    return readonly


class EngramBaseline:
    chunk_rows = 131072

    def __init__(self, identity, shapes, dtype, fds) -> None:
        self.identity, self.shapes, self.dtype, self._fds = identity, shapes, dtype, fds

    @property
    def byte_size(self) -> int:
        return sum(rows * width for rows, width in self.shapes.values()) * _bytes_per_value(self.dtype)

    def __getstate__(self):  # processes receive duplicated descriptors
        return self.identity, self.shapes, self.dtype, {name: DupFd(fd) for name, fd in self._fds.items()}

    def __setstate__(self, state):
        identity, shapes, dtype, handles = state
        self.__init__(identity, shapes, dtype, {name: handle.detach() for name, handle in handles.items()})

    def __del__(self):
        for fd in getattr(self, "_fds", {}).values():
            try:
                os.close(fd)
            except OSError:
                pass

    def view(self, name: str) -> torch.Tensor:
        """A private copy-on-write mapping of one table."""
        rows, width = self.shapes[name]
        pages = mmap.mmap(self._fds[name], rows * width * _bytes_per_value(self.dtype), access=mmap.ACCESS_COPY)
        return torch.frombuffer(pages, dtype=self.dtype).reshape(rows, width)

    @classmethod
    def create(cls, model_dir, config, dtype, random_init: bool, seed: int, initial_delta=None) -> "EngramBaseline":
        """Fill every table (seeded random init, released FP8 rows or native tensors), apply an
        optional initial delta, then seal."""
        from ..models.dsv4.checkpoint import ShardedSafeTensorReader
        from .checkpoint import file_sha256

        root = Path(model_dir)
        identity = baseline_identity(root, config, dtype, random_init, seed)
        shapes = {name: tuple(shape) for name, shape in identity["tables"].items()}
        if not shapes or dtype not in (torch.float32, torch.bfloat16):
            raise ValueError("trainable Engram requires nonempty FP32 or BF16 CPU tables")
        delta = None
        if initial_delta is not None:
            delta = torch.load(initial_delta, map_location="cpu", weights_only=True)
            validate_delta(delta, identity, shapes, dtype)
            identity = {**identity, "initial_delta_sha256": file_sha256(initial_delta)}
        sealed = sys.platform == "linux"
        itemsize = _bytes_per_value(dtype)
        if not sealed and sum(r * w for r, w in shapes.values()) * itemsize > _FALLBACK_LIMIT:
            raise RuntimeError("large Engram baselines require Linux memfd")
        reader = None if random_init else ShardedSafeTensorReader(root)
        source = _TableSource(reader, config, reader is not None and getattr(config, "checkpoint_format", "native")
                              == "released", random_init, seed)
        fds: dict[str, int] = {}
        try:
            for name, (rows, width) in shapes.items():
                size = rows * width * itemsize
                fd, path = _new_table_file(name, size, sealed)
                fds[name] = fd
                pages = mmap.mmap(fd, size, access=mmap.ACCESS_WRITE)
                try:
                    table = torch.frombuffer(pages, dtype=dtype).reshape(rows, width)
                    source.fill(name, table, cls.chunk_rows)
                    if delta is not None:
                        record = delta["tables"][name]
                        table.index_copy_(0, record["indices"], record["values"])
                    del table
                finally:
                    pages.close()
                    if path is not None:
                        fds[name] = _freeze_fallback(fd, path)
                if sealed:
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
    """A role's private view of one table, looked up from host memory; results land on the
    device of the ``placement`` buffer (which follows ``.to()`` / ``.cuda()`` of the model)."""

    sparse_gradients = engram_offload = True

    def __init__(self, weight: torch.Tensor, trainable: bool) -> None:
        super().__init__()
        self.weight = nn.Parameter(weight, requires_grad=trainable)
        self.register_buffer("placement", torch.empty(0, dtype=weight.dtype), persistent=False)
        self._cpu_lookup = CPUEmbeddingLookup()

    def _apply(self, fn, recurse=True):
        # the table itself stays in host memory; only the placement moves
        moved = fn(self.placement)
        if moved.dtype != self.weight.dtype:
            raise ValueError("Engram baseline dtype is fixed; build it in the training dtype")
        self.synchronize()
        self.placement = moved
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
        if role not in ROLES:
            raise ValueError("unknown Engram policy role")
        self.baseline, self.role = baseline, role
        learner = trainable and role == "learner"
        self.tables = {name: RoleEmbedding(baseline.view(name), learner) for name in baseline.shapes}
        self.dirty = {name: torch.empty(0, dtype=torch.long) for name in self.tables}

    @property
    def byte_size(self) -> int:
        return self.baseline.byte_size

    def synchronize(self) -> None:
        for table in self.tables.values():
            table.synchronize()

    def mark_touched(self) -> None:
        """Add the rows of the current sparse gradients to the learner's touched set."""
        if self.role != "learner":
            raise RuntimeError("only the learner may update Engram")
        for name, table in self.tables.items():
            grad = table.weight.grad
            if grad is None:
                continue
            if not grad.is_sparse:
                raise ValueError("Engram gradients must be sparse")
            touched = grad.coalesce().indices()[0]
            self.dirty[name] = torch.cat((self.dirty[name], touched)).unique(sorted=True)

    def state_dict(self) -> dict:
        self.synchronize()
        tables = {}
        for name, rows in self.dirty.items():
            tables[name] = {"indices": rows.clone(), "values": self.tables[name].weight.detach().index_select(0, rows)}
        return {"format": 1, "base": deepcopy(self.baseline.identity), "tables": tables}

    def validate(self, payload) -> None:
        if self.role == "reference":
            raise ValueError("the initial reference cannot load learner Engram state")
        validate_delta(payload, self.baseline.identity, self.baseline.shapes, self.baseline.dtype)

    @torch.no_grad()
    def load_state_dict(self, payload) -> None:
        self.validate(payload)
        self.synchronize()
        for name, table in self.tables.items():
            pristine = self.baseline.view(name)
            for rows in self.dirty[name].split(self.baseline.chunk_rows):  # back to the baseline first
                table.weight.index_copy_(0, rows, pristine.index_select(0, rows))
            record = payload["tables"][name]
            table.weight.index_copy_(0, record["indices"], record["values"])
            table.weight.grad = None
            self.dirty[name] = record["indices"].clone()
            table.clear_cache()


__all__ = ["EngramBaseline", "EngramState", "RoleEmbedding", "baseline_identity", "create_memfd", "memfd_seals",
           "seal_memfd", "validate_delta"]
