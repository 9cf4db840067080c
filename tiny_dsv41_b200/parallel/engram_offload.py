"""Engram tables kept in host memory, served to the GPU through a direct-mapped row cache.

Behaviour matched: ``dsv41_train/engram_offload.py:9-386`` (``_RowCache`` 29-203,
``CPUEmbeddingLookup`` 206-334, ``install_engram_sgd_hooks`` 337-386).

Data flow of one cached lookup (``RowCache.read``), all on the caller's stream unless noted:

1. The cache is bound to the table it serves. A different tensor, a moved or reshaped storage or
   a new ``_version`` (an in-place update such as an SGD step) invalidates every slot, so stale rows
   are never served.
2. Slot of a row id = id mod capacity; int64 tags live on the host. Hits are gathered into the
   output first, before any slot is rewritten in this lookup.
3. The distinct missing ids are gathered on the host into a pinned staging buffer (at most 4 MiB,
   or one row when a row is larger) and copied to a device staging buffer on a side stream. Only
   one such transfer is outstanding; its ticket carries the cache generation, the table's identity
   and version, and the copy's completion event, and is refused if any of them changed. The host
   rewrites the pinned buffer only after the previous copy out of it completed, and the side stream
   overwrites the device staging buffer only after the previous consumer finished reading it.
4. Every missing occurrence takes its row from the staging buffer (never from a slot, which
   another id of the same lookup may claim). Then each slot touched by the chunk is given exactly
   one id - the last distinct id that maps to it - and the tags follow the stored rows.

Outputs are independent copies, so rows a later lookup evicts stay valid for backward. The
backward is a sparse COO gradient on the host that keeps every occurrence in request order; the
table's accumulation hook concatenates micro-batches instead of summing them in low precision,
and :func:`install_engram_sgd_hooks` coalesces once in fp32 before ``torch.optim.SGD.step`` and
invalidates the caches after it.
"""

from __future__ import annotations

import weakref
from dataclasses import dataclass

import torch
import torch.nn.functional as F

_EMPTY_METRICS = dict(hits=0, misses=0, transferred_rows=0, resident_bytes=0)


class _CachedRows(torch.autograd.Function):
    @staticmethod
    def forward(ctx, weight, indices, cache):
        ids = indices.reshape(-1).long()
        ctx.save_for_backward(ids)
        ctx.table_shape = weight.shape
        return cache.read(weight, ids).view(*indices.shape, weight.shape[1])

    @staticmethod
    def backward(ctx, grad):
        (ids,) = ctx.saved_tensors
        values = grad.reshape(-1, ctx.table_shape[1]).to("cpu")
        sparse = torch.sparse_coo_tensor(ids.unsqueeze(0), values, ctx.table_shape, is_coalesced=False,
                                         check_invariants=False)
        return sparse, None, None


@dataclass
class _Ticket:
    """One host-to-device row transfer in flight."""

    generation: int
    table: tuple
    version: int
    rows: int
    ready: object  # torch.cuda.Event, or None on the CPU path


def _table_key(weight: torch.Tensor) -> tuple:
    return (id(weight), weight.data_ptr(), weight.untyped_storage().data_ptr(), tuple(weight.shape),
            tuple(weight.stride()), weight.dtype)


def _slot_owners(slots: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """For slot numbers of distinct ids in id order, the distinct slots and, for each, the position
    of the last id that maps to it (that id keeps the slot)."""
    order = torch.argsort(slots, stable=True)
    ordered = slots[order]
    last = torch.ones_like(ordered, dtype=torch.bool)
    last[:-1] = ordered[1:] != ordered[:-1]
    return ordered[last], order[last]


class RowCache:
    """Direct-mapped cache of one table's rows on ``device`` within ``budget`` bytes (the int64
    host tags count against the budget; the staging buffers and outputs do not)."""

    STAGING_BYTES = 4 * 2 ** 20

    def __init__(self, budget: int, device: torch.device) -> None:
        self.budget = budget
        self.device = device
        self.metrics = dict(_EMPTY_METRICS)
        self.values: torch.Tensor | None = None
        self.tags: torch.Tensor | None = None
        self._table: tuple | None = None
        self._table_ref = None
        self._version: int | None = None
        self._generation = 0
        self._ticket: _Ticket | None = None
        self._pinned = self._staging = self._stream = None
        self._copied = self._consumed = self._last_use = None

    # -- ownership and invalidation -------------------------------------------------------------
    def drain(self) -> None:
        """Wait for every copy and read this cache issued."""
        for event in (self._copied, self._consumed, self._last_use):
            if event is not None:
                event.synchronize()
        self._copied = self._consumed = self._last_use = None
        self._ticket = None

    def invalidate(self) -> None:
        self._generation += 1
        self.drain()
        if self.tags is not None:
            self.tags.fill_(-1)
        self._version = None

    def _bind(self, weight: torch.Tensor) -> None:
        key = _table_key(weight)
        same = self._table == key and self._table_ref is not None and self._table_ref() is weight
        if not same:
            width = weight.shape[1]
            capacity = min(weight.shape[0], self.budget // (width * weight.element_size() + 8))
            if capacity < 1:
                raise ValueError("Engram cache budget must hold one complete row and its int64 tag")
            self.invalidate()
            # release the old generation before allocating the new one: never two inside the budget
            self.values = self.tags = self._pinned = self._staging = None
            with torch.inference_mode(False), torch.no_grad():
                self.values = torch.empty(capacity, width, dtype=weight.dtype, device=self.device)
                self.tags = torch.full((capacity,), -1, dtype=torch.long)
            self.metrics["resident_bytes"] = capacity * (width * weight.element_size() + 8)
            self._table, self._table_ref = key, weakref.ref(weight)
            self._version = weight._version
        elif weight._version != self._version:
            self.invalidate()
            self._version = weight._version

    # -- staged transfers -----------------------------------------------------------------------
    def _chunk_rows(self, weight: torch.Tensor) -> int:
        return max(1, min(self.budget, self.STAGING_BYTES) // (weight.shape[1] * weight.element_size()))

    def _begin(self, weight: torch.Tensor, ids: torch.Tensor) -> _Ticket:
        if self._ticket is not None:
            raise RuntimeError("Engram cache allows one outstanding row transfer")
        n = ids.numel()
        self.metrics["transferred_rows"] += n
        if self.device.type != "cuda":
            self._staging = weight.detach().index_select(0, ids)
            self._ticket = _Ticket(self._generation, self._table, weight._version, n, None)
            return self._ticket
        if self._pinned is None:
            rows = self._chunk_rows(weight)
            self._stream = self._stream or torch.cuda.Stream(self.device)
            with torch.inference_mode(False), torch.no_grad():
                self._pinned = torch.empty(rows, weight.shape[1], dtype=weight.dtype, pin_memory=True)
                self._staging = torch.empty(rows, weight.shape[1], dtype=weight.dtype, device=self.device)
        if n > self._pinned.shape[0]:
            raise ValueError("Engram transfer exceeds the staging buffer")
        if self._copied is not None:  # the previous copy out of the pinned rows must be done
            self._copied.synchronize()
        torch.index_select(weight.detach(), 0, ids, out=self._pinned[:n])
        with torch.cuda.stream(self._stream):
            if self._consumed is not None:  # the previous reader of the staging rows must be done
                self._stream.wait_event(self._consumed)
            self._staging[:n].copy_(self._pinned[:n], non_blocking=True)
            ready = torch.cuda.Event()
            ready.record(self._stream)
        self._copied = ready
        self._ticket = _Ticket(self._generation, self._table, weight._version, n, ready)
        return self._ticket

    def _claim(self, weight: torch.Tensor, ticket: _Ticket) -> torch.Tensor:
        valid = (ticket is self._ticket and ticket.generation == self._generation
                 and ticket.table == _table_key(weight) and ticket.version == weight._version)
        if not valid:
            if ticket.ready is not None:
                ticket.ready.synchronize()
            if ticket is self._ticket:
                self._ticket = None
            raise RuntimeError("Engram table changed during a lookup; run a fresh forward")
        if ticket.ready is not None:
            consumer = torch.cuda.current_stream(self.device)
            consumer.wait_event(ticket.ready)
            self._staging.record_stream(consumer)
        return self._staging[:ticket.rows]

    def _end(self) -> None:
        if self.device.type == "cuda":
            self._consumed = torch.cuda.Event()
            self._consumed.record(torch.cuda.current_stream(self.device))
        self._ticket = None

    # -- lookup ---------------------------------------------------------------------------------
    def read(self, weight: torch.Tensor, ids: torch.Tensor) -> torch.Tensor:
        on_gpu = self.device.type == "cuda"
        if on_gpu and self._last_use is not None:
            torch.cuda.current_stream(self.device).wait_event(self._last_use)
        self._bind(weight)
        if ids.numel() and (int(ids.min()) < 0 or int(ids.max()) >= weight.shape[0]):
            raise IndexError("Engram row id outside the table")
        if on_gpu:
            self.values.record_stream(torch.cuda.current_stream(self.device))
        capacity = self.tags.numel()
        out = torch.empty(ids.numel(), weight.shape[1], dtype=weight.dtype, device=self.device)
        try:
            slots = ids.remainder(capacity)
            hit = self.tags[slots] == ids
            hit_pos = hit.nonzero().flatten()
            miss_pos = (~hit).nonzero().flatten()
            self.metrics["hits"] += hit_pos.numel()
            self.metrics["misses"] += miss_pos.numel()
            if hit_pos.numel():
                out.index_copy_(0, hit_pos.to(self.device),
                                self.values.index_select(0, slots[hit_pos].to(self.device)))
            if miss_pos.numel():
                self._serve_misses(weight, ids[miss_pos], miss_pos, out)
        except Exception:
            self.tags.fill_(-1)
            self._version = None
            raise
        finally:
            if on_gpu:
                self._last_use = torch.cuda.Event()
                self._last_use.record(torch.cuda.current_stream(self.device))
        return out

    def _serve_misses(self, weight, miss_ids, miss_pos, out) -> None:
        distinct, which = miss_ids.unique(sorted=True, return_inverse=True)
        capacity = self.tags.numel()
        step = self._chunk_rows(weight)
        for start in range(0, distinct.numel(), step):
            chunk = distinct[start:start + step]
            in_chunk = ((which >= start) & (which < start + chunk.numel())).nonzero().flatten()
            slots, owners = _slot_owners(chunk.remainder(capacity))
            ticket = self._begin(weight, chunk)
            try:
                rows = self._claim(weight, ticket)
                dev = lambda t: t.to(self.device, non_blocking=True)  # noqa: E731
                out.index_copy_(0, dev(miss_pos[in_chunk]), rows.index_select(0, dev(which[in_chunk] - start)))
                self.values.index_copy_(0, dev(slots), rows.index_select(0, dev(owners)))
                self.tags[slots] = chunk[owners]
            finally:
                self._end()


class CPUEmbeddingLookup:
    """Serves rows of a host-resident table on the caller's device, optionally through a
    :class:`RowCache`. One lookup per table per backward; micro-batch gradients are kept as
    concatenated occurrences until the SGD hook coalesces them in fp32."""

    def __init__(self) -> None:
        self._cache: RowCache | None = None
        self._hooked = None  # weakref to the parameter carrying the accumulation hook
        self._hook = None
        self._pending = 0

    def configure_cache(self, budget_bytes: int, device) -> None:
        """Per-table budget in bytes (tags included); 0 serves rows without a cache. Resets the
        counters."""
        if type(budget_bytes) is not int or budget_bytes < 0:
            raise ValueError("Engram cache budget must be a nonnegative integer")
        device = torch.device(device)
        if device.type not in ("cpu", "cuda"):
            raise ValueError("Engram cache runs on the CPU (tests) or a CUDA device")
        if device.type == "cuda" and device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        if self._cache is not None:
            self._cache.drain()
        self._cache = RowCache(budget_bytes, device) if budget_bytes else None

    def clear_cache(self) -> None:
        """Invalidate the cached rows (also needed after writes through ``.data``, which do not
        bump the tensor version)."""
        if self._cache is not None:
            self._cache.invalidate()

    def synchronize(self) -> None:
        if self._cache is not None:
            self._cache.drain()

    @property
    def cache_metrics(self) -> dict:
        return dict(self._cache.metrics) if self._cache is not None else dict(_EMPTY_METRICS)

    def __deepcopy__(self, memo):
        clone = type(self)()
        if self._cache is not None:
            clone.configure_cache(self._cache.budget, self._cache.device)
        return clone

    def _install_accumulation_hook(self, weight: torch.Tensor) -> None:
        if not (weight.requires_grad and weight.dtype in (torch.bfloat16, torch.float16)):
            return
        if self._hooked is not None and self._hooked() is weight:
            return
        if self._hook is not None:
            self._hook.remove()
        ref = weakref.ref(weight)

        def keep_occurrences(incoming):
            self._pending = 0
            param = ref()
            if param is None or param.grad is None:
                return incoming
            if not (incoming.is_sparse and param.grad.is_sparse):
                raise RuntimeError("offloaded Engram gradients must be sparse COO")
            merged = torch.sparse_coo_tensor(torch.cat((param.grad._indices(), incoming._indices()), 1),
                                             torch.cat((param.grad._values(), incoming._values())),
                                             incoming.shape, is_coalesced=False, check_invariants=False)
            param.grad = None  # the engine then stores `merged` instead of adding in low precision
            return merged

        self._hook = weight.register_hook(keep_occurrences)
        self._hooked = ref

    def __call__(self, weight: torch.Tensor, indices: torch.Tensor, *, device) -> torch.Tensor:
        if weight.device.type != "cpu":
            raise RuntimeError("offloaded Engram weights must stay on CPU")
        if indices.dtype not in (torch.int32, torch.int64):
            raise TypeError("Engram indices must be int32 or int64")
        device = torch.device(device)
        if device.type == "cuda" and device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        if self._cache is not None and device != self._cache.device:
            raise ValueError("Engram lookup device differs from the configured cache device")
        self._install_accumulation_hook(weight)
        self._pending = 0  # a fresh forward drops the count of an aborted backward
        cpu_ids = indices.to("cpu")
        if self._cache is not None:
            rows = _CachedRows.apply(weight, cpu_ids, self._cache)
        else:
            rows = F.embedding(cpu_ids, weight, sparse=True)
        if self._hook is not None and rows.requires_grad:
            # counted where the gradient flows, so a checkpoint recompute of the lookup is not a second use
            def count(grad):
                if self._pending:
                    raise RuntimeError("offloaded Engram allows one lookup per table per backward")
                self._pending = 1
                return grad

            rows.register_hook(count)
        return rows.to(device)


def install_engram_sgd_hooks(model, optimizer):
    """Coalesce sparse Engram gradients (fp32 accumulation) before SGD, invalidate caches after.

    Returns the two removable optimizer hook handles, or ``()`` when no table is trainable."""
    tables = [m for m in model.modules()
              if hasattr(m, "engram_offload") and getattr(m, "sparse_gradients", False) and m.weight.requires_grad]
    if not tables:
        return ()
    if type(optimizer) is not torch.optim.SGD:
        raise ValueError("trainable sparse Engram requires native torch.optim.SGD")
    owned = {id(p): g for g in optimizer.param_groups for p in g["params"]}
    for table in tables:
        group = owned.get(id(table.weight))
        if group is None:
            raise ValueError("optimizer does not own the Engram table")
        if any(group.get(k) for k in ("momentum", "weight_decay", "maximize", "foreach", "fused")):
            raise ValueError("sparse Engram SGD needs zero momentum and decay, foreach and fused off")

    def before(_opt, _args, _kwargs):
        for table in tables:
            table.synchronize()
            grad = table.weight.grad
            if grad is None:
                continue
            if not grad.is_sparse:
                raise RuntimeError("Engram SGD requires sparse COO gradients")
            low = grad.dtype in (torch.bfloat16, torch.float16)
            table.weight.grad = grad.float().coalesce().to(grad.dtype) if low else grad.coalesce()

    def after(_opt, _args, _kwargs):
        for table in tables:
            table.clear_cache()

    return optimizer.register_step_pre_hook(before), optimizer.register_step_post_hook(after)


__all__ = ["CPUEmbeddingLookup", "RowCache", "install_engram_sgd_hooks"]
