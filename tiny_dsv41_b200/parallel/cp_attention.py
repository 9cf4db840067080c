"""Context-parallel causal attention with the K/V exchange over NVLink peer memory instead of
an all-gather (fused path 3).

The reference gathers every rank's keys and values with an autograd all-gather and runs SDPA
with an explicit [L_local, L] mask (``dsv41_train/cp.py:17-35``, ``dsv41_train/models/qwen/
model.py:143-169``); the gather's backward is a reduce-scatter. Here:

* Each CP rank publishes its layer's K / V chunk into a symmetric buffer (one slot per layer,
  ``torch.distributed._symmetric_memory``), raises a ready flag and waits for its peers' flags.
* Causal attention needs only the chunks of lower ranks. This rank copies exactly those into a
  local staging buffer with its own peer-load kernel (``attn_cp_pull``: each remote byte crosses
  NVLink once per use, instead of once per query tile), and the tcgen05 attention kernels
  (``attn_fwd_cp`` / ``attn_bwd_cp`` in ``csrc/attention.cu``) walk the visible key tiles in
  global order, each tile taken by TMA from the chunk of its owner in local memory.
* The backward keeps dQ local and reduce-adds the dK / dV partials of every key owner into this
  rank's fp32 outbox (one slot per owner). After a flag exchange each owner sums its slot of all
  outboxes with peer loads in fixed rank order (``attn_cp_finalize``): the reduce-scatter of the
  reference, done by the attention backward's epilogue kernel, deterministic.

No kernel here issues a TMA load from another GPU's memory: an early version that streamed peer
K / V tiles by TMA straight into the softmax pipeline produced wrong outputs for tiles of V read
that way on B200 (the same bytes read with plain loads were correct), so remote data always lands
in local memory first.

Buffer reuse is guarded by epoch flags with bounded device waits (status 5 on timeout, raised by
the training loop's status monitor): a rank rewrites its K / V slot of a layer only after every
peer signalled that it finished reading the previous generation (after that layer's backward),
and zeroes its outbox only after every owner finished summing the previous one.

Activation checkpointing: the recompute of a layer (``parallel.replay`` mode ``replay``) re-pulls
the K / V its first forward published and exchanges no flag. A forward without autograd
(evaluation) releases its generation at once.

Semantics: plain causal attention over the concatenation of the ranks' equal contiguous chunks
(rank r holds positions [r * chunk, (r + 1) * chunk) of every sequence), bf16, head dim 128,
chunk a multiple of 128, at most 8 CP ranks. Other cases (padding masks, packed sequences, KV
caches) use the gather + masked attention path of :class:`~tiny_dsv41_b200.parallel.cp.ContextParallel`.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from .. import ops
from . import replay

_KV_READY, _KV_DONE = 0, 1  # per-layer flag rows (2 per layer), then the two outbox rows
_MAX_OWNERS = 8


class CPAttentionWorkspace:
    """Symmetric buffers and flags of one CP group: per-layer K / V slots, an fp32 outbox for
    dK / dV partials, and epoch flags."""

    def __init__(self, group, num_layers: int, batch: int, chunk: int, kv_heads: int, head_dim: int,
                 device: torch.device) -> None:
        import torch.distributed._symmetric_memory as symm

        self.group = group
        self.size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.size > _MAX_OWNERS:
            raise ValueError(f"fused CP attention supports at most {_MAX_OWNERS} ranks")
        self.num_layers, self.batch, self.chunk, self.kv_heads, self.head_dim = (num_layers, batch, chunk, kv_heads,
                                                                                  head_dim)
        self.device = device
        shape = (batch, chunk, kv_heads, head_dim)
        self.kv = symm.empty(num_layers, 2, *shape, dtype=torch.bfloat16, device=device)
        self.outbox = symm.empty(self.size, 2, *shape, dtype=torch.float32, device=device)
        rows = 2 * num_layers + 2
        self.flags = symm.empty(rows, self.size, dtype=torch.int32, device=device)
        self.flags.zero_()
        handles = {name: symm.rendezvous(getattr(self, name), group) for name in ("kv", "outbox", "flags")}
        torch.cuda.synchronize(device)
        dist.barrier(group=group)
        self._kv_bases = [int(p) for p in handles["kv"].buffer_ptrs]
        slot = self.kv[0].numel() * 2  # bytes of one layer slot (K and V)
        self._slot_bytes = slot
        self._half_bytes = slot // 2
        # local copies of the lower ranks' K / V chunks ([rank, 2, B, chunk, Hkv, 128]) and, per
        # layer, the table of their slots in those ranks' memory
        self.staging = torch.empty(max(self.rank, 1), 2, *shape, dtype=torch.bfloat16, device=device)
        self._pull_tables = [torch.tensor([base + layer * slot for base in self._kv_bases[:self.rank]],
                                          dtype=torch.int64, device=device) for layer in range(num_layers)]
        self.box_table = torch.tensor([int(p) for p in handles["outbox"].buffer_ptrs], dtype=torch.int64,
                                      device=device)
        self._flag_tables = [torch.tensor([int(p) + row * self.size * 4 for p in handles["flags"].buffer_ptrs],
                                          dtype=torch.int64, device=device) for row in range(rows)]
        self.kv_epoch = [0] * num_layers
        self.kv_released = [0] * num_layers
        self.box_epoch = 0
        self._handles = handles

    def matches(self, batch, chunk, kv_heads, head_dim) -> bool:
        return (batch, chunk, kv_heads, head_dim) == (self.batch, self.chunk, self.kv_heads, self.head_dim)

    # -- flags ----------------------------------------------------------------------------------
    def _row(self, layer: int, which: int) -> int:
        return 2 * layer + which

    def signal(self, row: int, epoch: int) -> None:
        ops.ext().ep_signal(self._flag_tables[row], None, None, self.rank, epoch)

    def wait(self, row: int, epoch: int) -> None:
        if epoch > 0:
            ops.ext().ep_wait(self.flags[row], epoch)

    # -- K / V slots ----------------------------------------------------------------------------
    def pull(self, layer: int) -> tuple[list[int], list[int]]:
        """Copy the lower ranks' K / V of `layer` into the staging buffer (peer loads); returns the
        local K and V addresses of every visible owner's chunk (owners 0 .. rank)."""
        if self.rank:
            ops.ext().attn_cp_pull(self._pull_tables[layer], self.staging, self._slot_bytes)
        staged = self.staging.data_ptr()
        k = [staged + c * self._slot_bytes for c in range(self.rank)] + [self.kv[layer, 0].data_ptr()]
        v = [p + self._half_bytes for p in k[:-1]] + [self.kv[layer, 1].data_ptr()]
        return k, v

    def publish(self, layer: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """Write this rank's K / V of `layer` into its slot once every peer has released the
        previous generation, then exchange ready flags."""
        epoch = self.kv_epoch[layer]
        self.wait(self._row(layer, _KV_DONE), epoch)
        self.kv[layer, 0].copy_(k)
        self.kv[layer, 1].copy_(v)
        self.kv_epoch[layer] = epoch + 1
        self.signal(self._row(layer, _KV_READY), epoch + 1)
        self.wait(self._row(layer, _KV_READY), epoch + 1)

    def release(self, layer: int) -> None:
        """This rank has finished reading every peer's K / V of `layer` (this generation)."""
        epoch = self.kv_epoch[layer]
        if self.kv_released[layer] < epoch:
            self.kv_released[layer] = epoch
            self.signal(self._row(layer, _KV_DONE), epoch)

    # -- outbox ---------------------------------------------------------------------------------
    def outbox_acquire(self) -> None:
        self.wait(2 * self.num_layers + 1, self.box_epoch)  # every owner summed the previous partials

    def outbox_exchange(self) -> tuple[torch.Tensor, torch.Tensor]:
        self.box_epoch += 1
        ready, done = 2 * self.num_layers, 2 * self.num_layers + 1
        self.signal(ready, self.box_epoch)
        self.wait(ready, self.box_epoch)
        dk, dv = ops.ext().attn_cp_finalize(self.box_table, self.rank, self.batch, self.chunk, self.kv_heads)
        self.signal(done, self.box_epoch)
        return dk, dv


class _CPAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, ws: CPAttentionWorkspace, layer: int):
        _, mode = replay.current()
        if mode != "replay":  # a recompute reads the generation its first forward published
            ws.publish(layer, k, v)
        kp, vp = ws.pull(layer)
        out, lse = ops.ext().attn_fwd_cp(q, kp, vp, ws.chunk, ws.rank * ws.chunk, ws.kv_heads)
        if not torch.is_grad_enabled() and mode is None:
            ws.release(layer)  # no backward follows
        ctx.ws, ctx.layer = ws, layer
        ctx.save_for_backward(q, out, lse)
        return out

    @staticmethod
    def backward(ctx, dout):
        ws, layer = ctx.ws, ctx.layer
        q, out, lse = ctx.saved_tensors
        kp, vp = ws.pull(layer)
        ws.release(layer)  # the peers' K / V of this generation are no longer read
        ws.outbox_acquire()
        dq = ops.ext().attn_bwd_cp(dout.contiguous(), q, kp, vp, out, lse, ws.chunk, ws.rank * ws.chunk, ws.kv_heads,
                                   ws.outbox)
        dk, dv = ws.outbox_exchange()
        return dq, dk, dv, None, None


def fused_supported(q: torch.Tensor, k: torch.Tensor, cp_size: int) -> bool:
    return (q.is_cuda and ops.available() and q.dtype == torch.bfloat16 and k.dtype == torch.bfloat16
            and q.shape[-1] == 128 and q.shape[1] % 128 == 0 and q.shape[1] > 0 and k.shape[1] == q.shape[1]
            and q.shape[2] % k.shape[2] == 0 and 1 < cp_size <= _MAX_OWNERS)


class FusedCPAttention:
    """Per-model owner of the workspace: ``__call__(q, k, v, layer)`` with this rank's chunk of
    q [B, chunk, H, 128] and k / v [B, chunk, Hkv, 128]."""

    def __init__(self, group, num_layers: int) -> None:
        self.group = group
        self.num_layers = num_layers
        self.ws: CPAttentionWorkspace | None = None

    def __call__(self, q, k, v, layer: int) -> torch.Tensor:
        batch, chunk, kv_heads, dim = k.shape
        if self.ws is None or not self.ws.matches(batch, chunk, kv_heads, dim):
            if self.ws is not None:
                raise ValueError("fused CP attention: the batch shape changed; one shape per workspace")
            self.ws = CPAttentionWorkspace(self.group, self.num_layers, batch, chunk, kv_heads, dim, q.device)
        return _CPAttention.apply(q.contiguous(), k.contiguous(), v.contiguous(), self.ws, layer)


__all__ = ["CPAttentionWorkspace", "FusedCPAttention", "fused_supported"]
