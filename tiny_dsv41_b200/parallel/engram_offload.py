"""Engram tables kept in host memory, with an optional direct-mapped row cache on the GPU.

Behaviour of ``dsv41_train/engram_offload.py``:

* :class:`CPUEmbeddingLookup` serves rows of a CPU-resident table to the caller's device. The
  backward produces a sparse COO gradient on the CPU that keeps every occurrence (duplicates and
  request order); one lookup per table per backward.
* With a cache budget the lookup first consults a direct-mapped GPU cache (slot = row % slots,
  int64 tags kept on the host); misses are copied through a pinned staging buffer of at most
  4 MiB on a side stream and then written into their slots. Metrics: hits, misses,
  transferred_rows, resident_bytes. The cache is invalidated after every optimizer step.
* :func:`install_engram_sgd_hooks` coalesces the sparse gradients of trainable tables in fp32
  before ``torch.optim.SGD.step`` and clears the caches afterwards.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


class _CachedRows(torch.autograd.Function):
    @staticmethod
    def forward(ctx, weight, indices, cache):
        ids = indices.reshape(-1).long()
        ctx.save_for_backward(ids)
        ctx.shape = weight.shape
        rows = cache.read(weight, ids)
        return rows.view(*indices.shape, weight.shape[1])

    @staticmethod
    def backward(ctx, grad):
        (ids,) = ctx.saved_tensors
        values = grad.reshape(-1, ctx.shape[1]).to("cpu")
        sparse = torch.sparse_coo_tensor(ids.unsqueeze(0), values, ctx.shape, is_coalesced=False,
                                         check_invariants=False)
        return sparse, None, None


class RowCache:
    """Direct-mapped cache of table rows on `device` within a byte budget (tags included)."""

    STAGING_BYTES = 4 * 2 ** 20

    def __init__(self, budget: int, device: torch.device) -> None:
        self.budget = budget
        self.device = device
        self.values: torch.Tensor | None = None
        self.tags: torch.Tensor | None = None
        self.signature = None
        self.metrics = dict(hits=0, misses=0, transferred_rows=0, resident_bytes=0)
        self._stream = None

    def clear(self) -> None:
        if self.tags is not None:
            self.tags.fill_(-1)

    def wait(self) -> None:
        if self._stream is not None:
            self._stream.synchronize()

    def _allocate(self, weight: torch.Tensor) -> None:
        signature = (weight.shape[1], weight.dtype)
        if self.signature == signature and self.values is not None:
            return
        row_bytes = weight.shape[1] * weight.element_size() + 8
        slots = max(0, min(self.budget // row_bytes, weight.shape[0]))
        self.values = torch.empty(slots, weight.shape[1], dtype=weight.dtype, device=self.device)
        self.tags = torch.full((slots,), -1, dtype=torch.long)
        self.signature = signature
        self.metrics["resident_bytes"] = slots * row_bytes

    def read(self, weight: torch.Tensor, ids: torch.Tensor) -> torch.Tensor:
        self._allocate(weight)
        slots = self.values.shape[0]
        if slots == 0:
            rows = weight.index_select(0, ids)
            self.metrics["misses"] += ids.numel()
            self.metrics["transferred_rows"] += ids.numel()
            return rows.to(self.device)
        slot = ids.remainder(slots)
        hit = self.tags[slot] == ids
        miss_ids = ids[~hit].unique()
        self.metrics["hits"] += int(hit.sum())
        self.metrics["misses"] += int((~hit).sum())
        if miss_ids.numel():
            self.metrics["transferred_rows"] += miss_ids.numel()
            self._fill(weight, miss_ids, slots)
        gpu_slots = slot.to(self.device, non_blocking=True)
        return self.values.index_select(0, gpu_slots)

    def _fill(self, weight: torch.Tensor, miss_ids: torch.Tensor, slots: int) -> None:
        row_bytes = weight.shape[1] * weight.element_size()
        chunk = max(1, self.STAGING_BYTES // row_bytes)
        # a later id that maps to the same slot wins; keep the last occurrence per slot
        target = miss_ids.remainder(slots)
        order = torch.argsort(target, stable=True)
        miss_ids, target = miss_ids[order], target[order]
        last = torch.ones_like(target, dtype=torch.bool)
        last[:-1] = target[1:] != target[:-1]
        miss_ids, target = miss_ids[last], target[last]
        if self.device.type == "cuda" and self._stream is None:
            self._stream = torch.cuda.Stream(self.device)
        for start in range(0, miss_ids.numel(), chunk):
            ids = miss_ids[start:start + chunk]
            slot = target[start:start + chunk]
            rows = weight.index_select(0, ids)
            if self.device.type == "cuda":
                rows = rows.pin_memory()
                with torch.cuda.stream(self._stream):
                    self.values.index_copy_(0, slot.to(self.device, non_blocking=True),
                                            rows.to(self.device, non_blocking=True))
                torch.cuda.current_stream(self.device).wait_stream(self._stream)
            else:
                self.values.index_copy_(0, slot, rows)
            self.tags[slot] = ids


class CPUEmbeddingLookup:
    def __init__(self) -> None:
        self._cache: RowCache | None = None

    def configure_cache(self, budget_bytes: int, device) -> None:
        if type(budget_bytes) is not int or budget_bytes < 0:
            raise ValueError("Engram cache budget must be a nonnegative integer")
        device = torch.device(device)
        if device.type == "cuda" and device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self._cache = RowCache(budget_bytes, device) if budget_bytes else None

    def clear_cache(self) -> None:
        if self._cache is not None:
            self._cache.clear()

    def synchronize(self) -> None:
        if self._cache is not None:
            self._cache.wait()

    @property
    def cache_metrics(self) -> dict:
        if self._cache is None:
            return dict(hits=0, misses=0, transferred_rows=0, resident_bytes=0)
        return dict(self._cache.metrics)

    def __call__(self, weight: torch.Tensor, indices: torch.Tensor, *, device) -> torch.Tensor:
        if weight.device.type != "cpu":
            raise RuntimeError("offloaded Engram weights must stay on CPU")
        if indices.dtype not in (torch.int32, torch.int64):
            raise TypeError("Engram indices must be int32 or int64")
        device = torch.device(device)
        cpu_indices = indices.to("cpu")
        if self._cache is not None:
            if device.type == "cuda" and device.index is None:
                device = torch.device("cuda", torch.cuda.current_device())
            if device != self._cache.device:
                raise ValueError("Engram lookup device differs from the configured cache device")
            return _CachedRows.apply(weight, cpu_indices, self._cache)
        rows = F.embedding(cpu_indices, weight, sparse=True)
        if device.type == "cuda":
            rows = rows.pin_memory() if not rows.requires_grad else rows
            return rows.to(device, non_blocking=True)
        return rows


def install_engram_sgd_hooks(model, optimizer):
    """Coalesce sparse Engram gradients (fp32 accumulation) before SGD, clear caches after."""
    tables = [m for m in model.modules()
              if hasattr(m, "engram_offload") and getattr(m, "sparse_gradients", False) and m.weight.requires_grad]
    if not tables:
        return ()
    if type(optimizer) is not torch.optim.SGD:
        raise ValueError("trainable sparse Engram requires native torch.optim.SGD")

    def before(_opt, _args, _kwargs):
        for table in tables:
            table.synchronize()
            grad = table.weight.grad
            if grad is None:
                continue
            if not grad.is_sparse:
                raise RuntimeError("Engram SGD requires sparse COO gradients")
            table.weight.grad = (grad.float().coalesce().to(grad.dtype)
                                 if grad.dtype in (torch.bfloat16, torch.float16) else grad.coalesce())

    def after(_opt, _args, _kwargs):
        for table in tables:
            table.clear_cache()

    return optimizer.register_step_pre_hook(before), optimizer.register_step_post_hook(after)


__all__ = ["CPUEmbeddingLookup", "RowCache", "install_engram_sgd_hooks"]
