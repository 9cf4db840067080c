"""Rebuild unsharded DeepSeek-V4.1 tensors from a complete full-SFT snapshot
(``dsv41_train/sft_source.py:23-259``): the initialization source for RL after SFT.

Each rank file of a same-topology snapshot holds local pieces: FSDP2 shards (dim-0 ``Shard`` of a
1-D mesh, pieces in mesh order), expert-parallel slices (``expert_start`` / ``num_experts`` of the
owning module), Engram row ranges (``row_start`` / ``row_stop``) or sparse Engram row snapshots.
The source validates the manifest, every rank digest, coverage (each element owned exactly once)
and dtypes before exposing anything, then copies tensors piecewise into caller-provided targets
(``copy_tensor``) - no full-model gather on one rank.
"""

from __future__ import annotations

import json
from pathlib import Path

import torch

from ..rl.checkpoint import file_sha256


def _owner_slice(name: str, ownership: dict):
    """(dim-0 offset, owner module record) for expert / Engram slices, else (0, None)."""
    for module, rec in ownership.items():
        if name.startswith(module + ".") and "expert_start" in rec and "num_experts" in rec:
            return rec["expert_start"], rec
        if name == f"{module}.weight" and "row_start" in rec:
            return rec["row_start"], rec
    return 0, None


class SFTCheckpointSource:
    def __init__(self, checkpoint, model_dir) -> None:
        from ..models.dsv4 import DeepSeekV41Config, DeepSeekV41ForCausalLM

        self.path = Path(checkpoint)
        manifest_path = self.path / "manifest.json"
        manifest = json.loads(manifest_path.read_text())
        world = manifest.get("world_size")
        if type(world) is not int or world < 1 or len(manifest.get("ranks", [])) != world or manifest.get("step", 0) < 1:
            raise ValueError("invalid complete SFT checkpoint manifest")
        config = DeepSeekV41Config.from_json(Path(model_dir) / "config.json")
        training = manifest["identity"].get("training_config", {})
        if training.get("family") != "dsv4" or training.get("mode") != "full" or \
                training.get("num_layers", config.num_hidden_layers) != config.num_hidden_layers:
            raise ValueError("SFT source requires complete-layer full DSV4 training")
        self.identity = {"manifest_sha256": file_sha256(manifest_path), "step": manifest["step"]}
        with torch.device("meta"):
            model = DeepSeekV41ForCausalLM(config)
        expected = model.state_dict()
        self.shapes = {n: tuple(v.shape) for n, v in expected.items()}
        self.dtypes: dict = {}
        self._pieces: dict[str, list] = {}  # name -> [(dim0 start, tensor)]
        self._rows: dict[str, list] = {}    # sparse Engram: name -> [(global ids, values)]
        for rank, record in enumerate(manifest["ranks"]):
            path = self.path / f"rank-{rank:05d}.pt"
            if file_sha256(path) != record["sha256"]:
                raise ValueError(f"SFT rank {rank} checksum differs")
            payload = torch.load(path, map_location="cpu", weights_only=False, mmap=True)
            schema = payload["schema"]
            ownership = schema["ownership"]
            values = {**payload["parameters"], **payload["buffers"]}
            layouts = {**schema["parameters"], **schema["buffers"]}
            for name, value in values.items():
                if name not in expected:
                    raise ValueError(f"unexpected SFT tensor {name}")
                layout = layouts[name]
                base, _ = _owner_slice(name, ownership)
                start = base
                if "mesh" in layout:
                    mesh = [r for row in layout["mesh"] for r in (row if isinstance(row, list) else [row])]
                    if not any(p in ("S(0)", "Shard(dim=0)") for p in layout["placements"]):
                        raise ValueError(f"unsupported SFT placement for {name}: {layout['placements']}")
                    position = mesh.index(rank)
                    # FSDP2 pads dim 0 to a multiple of the mesh size and gives rank i rows [i*c, (i+1)*c)
                    chunk = -(-layout["shape"][0] // len(mesh))
                    start = base + position * chunk
                self._add(name, start, value)
            rows = payload.get("engram_rows")
            if rows is not None:
                for name, rec in rows["tables"].items():
                    offset = rows["schema"][name]["row_start"]
                    self._rows.setdefault(name, []).append((rec["indices"] + offset, rec["values"]))
        self.tensor_names = set(self._pieces)
        for name in self.tensor_names:
            covered = sum(t.shape[0] if t.ndim else 1 for _, t in self._pieces[name])
            first = self.shapes[name][0] if self.shapes[name] else 1
            if covered < first:
                raise ValueError(f"SFT pieces do not cover {name} ({covered} of {first} rows)")

    def _add(self, name, start, value) -> None:
        dtype = self.dtypes.setdefault(name, value.dtype)
        if dtype != value.dtype:
            raise ValueError(f"inconsistent SFT dtype for {name}")
        self._pieces.setdefault(name, []).append((start, value))

    @torch.no_grad()
    def copy_tensor(self, name: str, target: torch.Tensor) -> None:
        if tuple(target.shape) != self.shapes[name]:
            raise ValueError(f"SFT target shape differs for {name}")
        if target.ndim == 0:
            target.copy_(self._pieces[name][0][1])
            return
        rows = target.shape[0]
        seen = torch.zeros(rows, dtype=torch.bool)
        for start, piece in sorted(self._pieces[name], key=lambda p: p[0]):
            stop = min(rows, start + piece.shape[0])
            if stop <= start:
                continue  # an FSDP padding-only shard
            if seen[start:stop].any() and not torch.equal(target[start:stop].cpu(), piece[:stop - start].to(target.dtype)):
                raise ValueError(f"SFT replicas of {name} disagree")
            target[start:stop].copy_(piece[:stop - start].to(device=target.device, dtype=target.dtype))
            seen[start:stop] = True
        if not bool(seen.all()):
            raise ValueError(f"SFT pieces leave rows of {name} uncovered")

    def iter_engram_rows(self, name: str):
        yield from self._rows.get(name, [])

    def state_dict(self) -> dict:
        out = {}
        for name in sorted(self.tensor_names):
            t = torch.empty(self.shapes[name], dtype=self.dtypes[name])
            self.copy_tensor(name, t)
            out[name] = t
        return out


__all__ = ["SFTCheckpointSource"]
