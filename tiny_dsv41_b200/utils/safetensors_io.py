"""Minimal safetensors reader/writer on the standard library (mmap), with row-slice reads.

Format: 8-byte little-endian header length, a JSON header ``{name: {dtype, shape, data_offsets},
"__metadata__": {...}}``, then the raw little-endian tensor bytes. Reading a row range touches
only those rows' pages, which is how expert ranges and Engram row shards are loaded without
reading whole tensors (same approach as ``dsv41_train/models/dsv4/checkpoint.py:31-190``).
"""

from __future__ import annotations

import json
import mmap
import struct
import warnings
from pathlib import Path

import torch

DTYPES = {
    "F64": torch.float64, "F32": torch.float32, "F16": torch.float16, "BF16": torch.bfloat16,
    "I64": torch.int64, "I32": torch.int32, "I16": torch.int16, "I8": torch.int8, "U8": torch.uint8,
    "BOOL": torch.bool, "F8_E4M3": torch.float8_e4m3fn, "F8_E5M2": torch.float8_e5m2,
}
if hasattr(torch, "float8_e8m0fnu"):
    DTYPES["F8_E8M0"] = torch.float8_e8m0fnu
NAMES = {v: k for k, v in DTYPES.items()}


class SafeTensorFile:
    def __init__(self, path) -> None:
        self.path = Path(path)
        self._file = self.path.open("rb")
        self._map = mmap.mmap(self._file.fileno(), 0, access=mmap.ACCESS_READ)
        (length,) = struct.unpack("<Q", self._map[:8])
        header = json.loads(self._map[8:8 + length])
        self.metadata_block = header.pop("__metadata__", {})
        self.header = header
        self.base = 8 + length

    def keys(self):
        return self.header.keys()

    def metadata(self, name: str) -> dict:
        return self.header[name]

    def _view(self, name: str, start_row: int | None = None, stop_row: int | None = None) -> torch.Tensor:
        info = self.header[name]
        dtype = DTYPES[info["dtype"]]
        shape = list(info["shape"])
        begin, end = info["data_offsets"]
        itemsize = torch.empty(0, dtype=dtype).element_size()
        if start_row is not None:
            row_bytes = itemsize * (int(torch.tensor(shape[1:]).prod().item()) if len(shape) > 1 else 1)
            begin, end = begin + start_row * row_bytes, begin + stop_row * row_bytes
            shape[0] = stop_row - start_row
        raw = memoryview(self._map)[self.base + begin:self.base + end]
        if end == begin:
            return torch.empty(shape, dtype=dtype)
        with warnings.catch_warnings():  # read-only map: callers copy (`tensor`) before any write
            warnings.simplefilter("ignore", UserWarning)
            return torch.frombuffer(raw, dtype=torch.uint8).view(dtype).reshape(shape)

    def tensor(self, name: str, device="cpu") -> torch.Tensor:
        return self._view(name).to(device, copy=True)

    def tensor_rows(self, name: str, start: int, stop: int, device="cpu") -> torch.Tensor:
        return self._view(name, start, stop).to(device, copy=True)

    def close(self) -> None:
        try:
            self._map.close()
        finally:
            self._file.close()


class ShardedSafeTensorReader:
    """Reads tensors of a sharded checkpoint through ``model.safetensors.index.json``."""

    def __init__(self, folder) -> None:
        self.folder = Path(folder)
        index = self.folder / "model.safetensors.index.json"
        if index.exists():
            self.weight_map = json.loads(index.read_text(encoding="utf-8"))["weight_map"]
        else:
            single = self.folder / "model.safetensors"
            self.weight_map = {k: single.name for k in SafeTensorFile(single).keys()}
        self._shards: dict[str, SafeTensorFile] = {}

    def _shard(self, name: str) -> SafeTensorFile:
        if name not in self.weight_map:
            raise KeyError(f"checkpoint has no tensor {name}")
        file = self.weight_map[name]
        if file not in self._shards:
            self._shards[file] = SafeTensorFile(self.folder / file)
        return self._shards[file]

    def __contains__(self, name: str) -> bool:
        return name in self.weight_map

    def metadata(self, name: str) -> dict:
        return self._shard(name).metadata(name)

    def tensor(self, name: str, device="cpu") -> torch.Tensor:
        return self._shard(name).tensor(name, device)

    def tensor_rows(self, name: str, start: int, stop: int, device="cpu") -> torch.Tensor:
        return self._shard(name).tensor_rows(name, start, stop, device)

    def close(self) -> None:
        for shard in self._shards.values():
            shard.close()
        self._shards.clear()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def save_file(tensors: dict[str, torch.Tensor], path, metadata: dict | None = None) -> None:
    header, offset, blobs = {}, 0, []
    for name, tensor in tensors.items():
        t = tensor.detach().contiguous().cpu()
        data = t.view(torch.uint8).numpy().tobytes() if t.numel() else b""
        header[name] = {"dtype": NAMES[t.dtype], "shape": list(t.shape), "data_offsets": [offset, offset + len(data)]}
        blobs.append(data)
        offset += len(data)
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    text = json.dumps(header).encode()
    text += b" " * (-len(text) % 8)
    with Path(path).open("wb") as f:
        f.write(struct.pack("<Q", len(text)))
        f.write(text)
        for blob in blobs:
            f.write(blob)


def save_sharded(tensors: dict[str, torch.Tensor], folder, shard_size: int = 2 ** 30) -> None:
    """Write tensors in shards plus ``model.safetensors.index.json``."""
    folder = Path(folder)
    folder.mkdir(parents=True, exist_ok=True)
    shards, current, size = [], {}, 0
    for name, t in tensors.items():
        nbytes = t.numel() * t.element_size()
        if current and size + nbytes > shard_size:
            shards.append(current)
            current, size = {}, 0
        current[name] = t
        size += nbytes
    if current:
        shards.append(current)
    weight_map = {}
    for i, shard in enumerate(shards):
        fname = f"model-{i + 1:05d}-of-{len(shards):05d}.safetensors"
        save_file(shard, folder / fname)
        weight_map.update({name: fname for name in shard})
    (folder / "model.safetensors.index.json").write_text(json.dumps({"metadata": {}, "weight_map": weight_map}))


__all__ = ["SafeTensorFile", "ShardedSafeTensorReader", "save_file", "save_sharded"]
