"""Direct LoRA update packets for an external vLLM rollout service.

Wire format of the reference service (``rollout_manager/backends/vllm_lora_transport.py:44-195``),
kept byte-compatible so the same service can load adapters trained here:

* payload: the raw little-endian bytes of each tensor, concatenated in sorted-name order;
* manifest (JSON, sorted keys, compact): ``schema_version`` 1, ``version``, ``lineage``,
  ``adapter_id`` (>= 1), ``peft`` ({r, lora_alpha, target_modules}), ``base_identity``,
  ``tensors`` (``name`` ending ``.lora_A.weight`` / ``.lora_B.weight``, 2-D ``shape``, ``dtype``
  float16 / bfloat16 / float32, contiguous ``offset`` / ``nbytes``, per-tensor ``sha256``),
  ``payload_sha256`` and ``digest`` = sha256(manifest-without-digest JSON + b"\\0" + payload);
* frame on a stream: ``struct.pack("!IQ", len(manifest), len(payload))`` + manifest + payload;
* budgets: 1 MiB manifest, 64 MiB payload, 128 tensors.

Validation checks every descriptor and byte before anything is applied.
"""

from __future__ import annotations

import hashlib
import json
import math
import re
import struct
import sys

MAX_MANIFEST_BYTES = 1 << 20
MAX_TENSOR_BYTES = 64 << 20
MAX_TENSORS = 128
_ITEMSIZE = {"float16": 2, "bfloat16": 2, "float32": 4}
_SHA = re.compile(r"[0-9a-f]{64}\Z")
_NAME = re.compile(r"[A-Za-z0-9_.]+\.lora_[AB]\.weight\Z")
_MANIFEST_KEYS = {"schema_version", "version", "lineage", "adapter_id", "peft", "base_identity", "tensors",
                  "payload_sha256", "digest"}
_TENSOR_KEYS = {"name", "shape", "dtype", "offset", "nbytes", "sha256"}


def _canonical(value) -> bytes:
    return json.dumps(value, sort_keys=True, separators=(",", ":"), allow_nan=False).encode()


def _packet_digest(manifest: dict, payload: bytes) -> str:
    body = {k: v for k, v in manifest.items() if k != "digest"}
    return hashlib.sha256(_canonical(body) + b"\x00" + payload).hexdigest()


def policy_ack(manifest: dict) -> dict:
    return {k: manifest[k] for k in ("version", "digest", "lineage")}


def validate_update(manifest, payload) -> dict:
    if sys.byteorder != "little":
        raise RuntimeError("direct LoRA tensor transport requires a little-endian host")
    schema_ok = (isinstance(manifest, dict) and set(manifest) == _MANIFEST_KEYS and manifest["schema_version"] == 1
                 and type(manifest["version"]) is int and manifest["version"] >= 0
                 and type(manifest["adapter_id"]) is int and manifest["adapter_id"] >= 1
                 and isinstance(manifest["lineage"], str) and 0 < len(manifest["lineage"]) <= 256
                 and isinstance(manifest["peft"], dict) and isinstance(manifest["base_identity"], dict)
                 and isinstance(payload, bytes) and 0 < len(payload) <= MAX_TENSOR_BYTES)
    if not schema_ok:
        raise ValueError("invalid direct LoRA update schema or byte budget")
    if len(_canonical(manifest)) > MAX_MANIFEST_BYTES:
        raise ValueError("direct LoRA manifest exceeds byte budget")
    tensors = manifest["tensors"]
    if not isinstance(tensors, list) or not 0 < len(tensors) <= MAX_TENSORS:
        raise ValueError("invalid direct LoRA tensor count")
    cursor, names = 0, []
    for item in tensors:
        if not isinstance(item, dict) or set(item) != _TENSOR_KEYS:
            raise ValueError("invalid direct LoRA tensor descriptor")
        shape, dtype = item["shape"], item["dtype"]
        ok = (isinstance(item["name"], str) and _NAME.fullmatch(item["name"]) and isinstance(shape, list)
              and len(shape) == 2 and all(type(n) is int and n >= 1 for n in shape) and dtype in _ITEMSIZE
              and type(item["offset"]) is int and type(item["nbytes"]) is int and item["offset"] == cursor
              and item["nbytes"] == math.prod(shape) * _ITEMSIZE[dtype]
              and isinstance(item["sha256"], str) and _SHA.fullmatch(item["sha256"]))
        if not ok:
            raise ValueError("invalid direct LoRA tensor shape, dtype, offset, or digest")
        cursor += item["nbytes"]
        if cursor > len(payload) or hashlib.sha256(payload[item["offset"]:cursor]).hexdigest() != item["sha256"]:
            raise ValueError("direct LoRA tensor bytes differ from manifest")
        names.append(item["name"])
    if names != sorted(set(names)) or cursor != len(payload):
        raise ValueError("direct LoRA tensors must be unique, sorted, and cover the payload")
    for key in ("payload_sha256", "digest"):
        if not isinstance(manifest[key], str) or not _SHA.fullmatch(manifest[key]):
            raise ValueError("invalid direct LoRA payload digest")
    if hashlib.sha256(payload).hexdigest() != manifest["payload_sha256"] or \
            _packet_digest(manifest, payload) != manifest["digest"]:
        raise ValueError("direct LoRA update digest mismatch")
    return manifest


def pack_update(tensors, *, version, lineage, adapter_id, peft, base_identity) -> tuple[dict, bytes]:
    """Snapshot finite CPU matrices into (manifest, payload); later trainer writes do not alias it."""
    import torch

    if not isinstance(tensors, dict) or not 0 < len(tensors) <= MAX_TENSORS:
        raise ValueError("a bounded nonempty adapter tensor dictionary is required")
    chunks, descriptors, offset = [], [], 0
    for name in sorted(tensors):
        t = tensors[name]
        if not isinstance(t, torch.Tensor):
            raise ValueError("LoRA values must be tensors")
        value = t.detach().cpu().contiguous()
        dtype = str(value.dtype).removeprefix("torch.")
        if dtype not in _ITEMSIZE or value.ndim != 2 or not bool(torch.isfinite(value).all()):
            raise ValueError("LoRA tensors must be finite matrices in a supported dtype")
        raw = value.view(torch.uint8).numpy().tobytes()
        if offset + len(raw) > MAX_TENSOR_BYTES:
            raise ValueError("direct LoRA tensors exceed byte budget")
        descriptors.append({"name": name, "shape": list(value.shape), "dtype": dtype, "offset": offset,
                            "nbytes": len(raw), "sha256": hashlib.sha256(raw).hexdigest()})
        chunks.append(raw)
        offset += len(raw)
    payload = b"".join(chunks)
    manifest = json.loads(_canonical({"schema_version": 1, "version": version, "lineage": lineage,
                                      "adapter_id": adapter_id, "peft": peft, "base_identity": base_identity,
                                      "tensors": descriptors, "payload_sha256": hashlib.sha256(payload).hexdigest()}))
    manifest["digest"] = _packet_digest(manifest, payload)
    validate_update(manifest, payload)
    return manifest, payload


def unpack_update(manifest, payload) -> dict:
    import torch

    validate_update(manifest, payload)
    out = {}
    for item in manifest["tensors"]:
        raw = bytearray(payload[item["offset"]:item["offset"] + item["nbytes"]])
        value = torch.frombuffer(raw, dtype=getattr(torch, item["dtype"])).reshape(item["shape"])
        if not bool(torch.isfinite(value).all()):
            raise ValueError("direct LoRA update contains nonfinite tensor values")
        out[item["name"]] = value
    return out


def _read_exact(stream, size: int) -> bytes:
    parts = []
    while size:
        part = stream.recv(size)
        if not part:
            raise EOFError("incomplete direct LoRA tensor frame")
        parts.append(part)
        size -= len(part)
    return b"".join(parts)


def send_update(stream, manifest, payload) -> None:
    validate_update(manifest, payload)
    meta = _canonical(manifest)
    stream.sendall(struct.pack("!IQ", len(meta), len(payload)) + meta + payload)


def receive_update(stream) -> tuple[dict, bytes]:
    meta_size, payload_size = struct.unpack("!IQ", _read_exact(stream, 12))
    if not 0 < meta_size <= MAX_MANIFEST_BYTES or not 0 < payload_size <= MAX_TENSOR_BYTES:
        raise ValueError("direct LoRA frame exceeds byte budget")
    manifest = json.loads(_read_exact(stream, meta_size))
    payload = _read_exact(stream, payload_size)
    validate_update(manifest, payload)
    return manifest, payload


__all__ = ["pack_update", "policy_ack", "receive_update", "send_update", "unpack_update", "validate_update"]
