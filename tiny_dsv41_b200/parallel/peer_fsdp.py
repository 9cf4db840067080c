"""Dense-parameter data parallelism over NVLink peer memory (fused path 2).

FSDP2 (what the reference uses, ``dsv41_train/models/qwen/parallel.py:28-45``) shards the bf16
weights and runs, per layer and step, an all-gather before the forward, a second one before the
backward (or keeps the layer gathered), an fp32 reduce-scatter of the gradients and then the
optimizer on the shard (``dsv41_train/optim.py:85-137``). On a B200 the dense weights of the
MoE models are small against 180 GB of HBM (3.1 GB in bf16 for Qwen3-30B-A3B), so this module
keeps them replicated in bf16 and shards only what is large: the fp32 master and the moments.

* The bf16 parameters of all units live in one symmetric buffer (the parameter pool; every
  parameter's ``.data`` is a view into it) and their gradients are staged in a second one.
* A unit is a group of parameters that becomes ready together in backward (one decoder layer,
  the embedding, the head). When the last gradient of a unit has been staged, one kernel
  (``csrc/peer_optim.cu::peer_update``) reads the rank's owned slice of the unit's gradient from
  every rank over NVLink, sums it in fp32 in rank order, applies AdamW or SGD to the owned fp32
  master and moments, and stores the rounded bf16 result into every rank's parameter pool. No
  all-gather runs in the forward pass, and the reduce-scatter, cast / scale, update and gather
  are one launch that runs on a side stream while the backward continues.
* ``finish_step()`` ends a step with a device-side barrier over a symmetric flag array, so the
  next forward reads parameters that every rank has finished writing and no rank re-stages a
  gradient a peer is still reading.

Unit kernels are enqueued in one fixed order on every rank (the order of ``units`` reversed, the
order in which backward produces them); a unit that completes early waits for its predecessors.
The step count and the flag epoch live in device memory (advanced by ``begin_step``), so a CUDA
graph captured over a training step replays with fresh epochs and bias corrections.

Without CUDA (gloo ranks on CPU, the test-suite) the same bookkeeping runs with an all-reduce
and an all-gather in place of the kernel.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Sequence

import torch
import torch.distributed as dist
from torch import nn

_ALIGN = 8  # elements: every parameter view and shard starts on a 16-byte boundary


@dataclass
class _Unit:
    index: int
    params: list
    offsets: list          # element offset of each parameter in the pools
    start: int             # first element of the unit in the pools
    shard: int             # elements owned per rank (multiple of _ALIGN)
    pending: int = 0
    staged: set = field(default_factory=set)
    launched: bool = False


def plan_units(sizes: Sequence[Sequence[int]], world: int) -> tuple[list[tuple[list[int], int, int]], int]:
    """Pool layout for units of parameters with the given element counts: per unit the offsets of
    its parameters, its start and its per-rank shard length; and the total pool length. Every
    offset and shard is a multiple of 8 elements and each unit spans ``world * shard`` elements."""
    layout, cursor = [], 0
    for unit_sizes in sizes:
        start, offsets, pos = cursor, [], cursor
        for n in unit_sizes:
            offsets.append(pos)
            pos += math.ceil(n / _ALIGN) * _ALIGN
        span = pos - start
        shard = math.ceil(span / (world * _ALIGN)) * _ALIGN if span else _ALIGN
        layout.append((offsets, start, shard))
        cursor = start + shard * world
    return layout, cursor


class PeerShardedOptimizer:
    """Replicated bf16 dense parameters with a sharded fp32 master and optimizer state.

    ``units``: groups of parameters (each parameter in one unit). ``algo``: ``"adamw"``
    (torch.optim.AdamW semantics) or ``"sgd"``. Gradients of all ranks are averaged
    (``grad_scale`` defaults to 1 / world). Call ``begin_step()`` before the backward of each step
    and ``finish_step()`` after it."""

    def __init__(self, units: Sequence[Sequence[nn.Parameter]], group=None, *, algo: str = "adamw",
                 lr: float = 1e-4, betas=(0.9, 0.999), eps: float = 1e-8, weight_decay: float = 0.0,
                 moment_dtype: torch.dtype = torch.float32, grad_scale: float | None = None,
                 max_blocks: int = 64) -> None:
        if algo not in ("adamw", "sgd"):
            raise ValueError(f"algo must be 'adamw' or 'sgd', not {algo!r}")
        self.group = group
        self.distributed = dist.is_initialized()
        self.world = dist.get_world_size(group) if self.distributed else 1
        self.rank = dist.get_rank(group) if self.distributed else 0
        self.algo = algo
        self.lr, self.betas, self.eps, self.weight_decay = lr, betas, eps, weight_decay
        self.grad_scale = 1.0 / self.world if grad_scale is None else grad_scale
        self.max_blocks = max_blocks
        self.step_count = 0
        self.epoch = 0
        units = [[p for p in u if p.requires_grad] for u in units]
        units = [u for u in units if u]
        seen = set()
        for u in units:
            for p in u:
                if id(p) in seen:
                    raise ValueError("a parameter appears in two units")
                seen.add(id(p))
        layout, total = plan_units([[p.numel() for p in u] for u in units], self.world)
        device = units[0][0].device
        self.device = device
        self.cuda = device.type == "cuda"
        dtype = units[0][0].dtype
        if self.cuda and dtype != torch.bfloat16:
            raise ValueError("the peer-memory path keeps bf16 parameters")
        self._alloc_pools(total, dtype, device, len(units))
        self.units: list[_Unit] = []
        self._unit_of: dict[int, tuple[_Unit, int]] = {}
        with torch.no_grad():
            for i, (params, (offsets, start, shard)) in enumerate(zip(units, layout)):
                unit = _Unit(i, list(params), offsets, start, shard)
                for j, (p, off) in enumerate(zip(params, offsets)):
                    view = self.param_pool[off:off + p.numel()].view(p.shape)
                    view.copy_(p.data)
                    p.data = view
                    self._unit_of[id(p)] = (unit, j)
                self.units.append(unit)
            if self.distributed:  # every replica starts from rank 0's values
                dist.broadcast(self.param_pool, src=dist.get_global_rank(group, 0) if group is not None else 0,
                               group=group)
        self.state = []
        for unit in self.units:
            lo = unit.start + self.rank * unit.shard
            master = self.param_pool[lo:lo + unit.shard].float().clone()
            st = {"master": master}
            if algo == "adamw":
                st["m"] = torch.zeros(unit.shard, dtype=moment_dtype, device=device)
                st["v"] = torch.zeros(unit.shard, dtype=moment_dtype, device=device)
            self.state.append(st)
        self.order = list(reversed(self.units))  # the order backward completes them
        self._next = 0
        self.nonfinite = torch.zeros(1, dtype=torch.int32, device=device)
        # device copies of the step count (bias corrections; restored with the state) and of the flag
        # epoch (only ever grows: the flags of earlier steps still hold their epochs)
        self._step_t = torch.zeros(1, dtype=torch.int32, device=device) if self.cuda else None
        self._epoch_t = torch.zeros(1, dtype=torch.int32, device=device) if self.cuda else None
        self.stream = torch.cuda.Stream(device=device) if self.cuda else None
        self._hooks = [p.register_post_accumulate_grad_hook(self._hook) for u in self.units for p in u.params]

    # -- pools ---------------------------------------------------------------------------------
    def _alloc_pools(self, total: int, dtype, device, n_units: int) -> None:
        self.flag_rows = n_units + 1  # one row per unit, the last one for the end-of-step barrier
        if not self.cuda:
            self.param_pool = torch.zeros(total, dtype=dtype, device=device)
            self.grad_pool = torch.zeros(total, dtype=dtype, device=device)
            return
        world = self.world
        if self.distributed and world > 1:
            import torch.distributed._symmetric_memory as symm

            self.param_pool = symm.empty(total, dtype=dtype, device=device)
            self.grad_pool = symm.empty(total, dtype=dtype, device=device)
            self.flags = symm.empty(self.flag_rows, world, dtype=torch.int32, device=device)
            self.flags.zero_()
            self.param_pool.zero_()
            self.grad_pool.zero_()
            handles = [symm.rendezvous(t, self.group if self.group is not None else dist.group.WORLD)
                       for t in (self.param_pool, self.grad_pool, self.flags)]
            torch.cuda.synchronize(device)
            dist.barrier(group=self.group)
            ptrs = [[int(x) for x in h.buffer_ptrs] for h in handles]
        else:
            self.param_pool = torch.zeros(total, dtype=dtype, device=device)
            self.grad_pool = torch.zeros(total, dtype=dtype, device=device)
            self.flags = torch.zeros(self.flag_rows, world, dtype=torch.int32, device=device)
            ptrs = [[t.data_ptr()] for t in (self.param_pool, self.grad_pool, self.flags)]
        self.peer_param = torch.tensor(ptrs[0], dtype=torch.int64)
        self.peer_grad = torch.tensor(ptrs[1], dtype=torch.int64)
        self.peer_flags = torch.tensor(ptrs[2], dtype=torch.int64)
        barrier_row = (self.flag_rows - 1) * world * 4
        self.peer_barrier = torch.tensor([p + barrier_row for p in ptrs[2]], dtype=torch.int64, device=device)

    # -- step protocol -------------------------------------------------------------------------
    def begin_step(self) -> None:
        self.step_count += 1
        self.epoch += 1
        if self._step_t is not None:
            self._step_t.add_(1)
            self._epoch_t.add_(1)
        self._next = 0
        for unit in self.units:
            unit.pending = len(unit.params)
            unit.staged = set()
            unit.launched = False

    def finish_step(self) -> None:
        """Launch the units whose gradients never arrived (their staged gradient is zero), then
        order the next step after every rank's updates (device-side barrier)."""
        for unit in self.order:
            if unit.pending:
                with torch.no_grad():
                    for j, (p, off) in enumerate(zip(unit.params, unit.offsets)):
                        if j not in unit.staged:
                            self.grad_pool[off:off + p.numel()].zero_()
                unit.pending = 0
        self._launch_ready()
        if not self.cuda:
            return
        from ..ops import ext

        C = ext()
        with torch.cuda.stream(self.stream):
            if self.world > 1:
                C.ep_signal(self.peer_barrier, None, None, self.rank, 0, self._epoch_t)
                C.ep_wait(self.flags[self.flag_rows - 1], 0, self._epoch_t)
        torch.cuda.current_stream(self.device).wait_stream(self.stream)

    def remove_hooks(self) -> None:
        for h in self._hooks:
            h.remove()
        self._hooks = []

    def zero_grad(self, set_to_none: bool = True) -> None:
        for unit in self.units:
            for p in unit.params:
                p.grad = None

    # -- internals -----------------------------------------------------------------------------
    def _hook(self, p: torch.Tensor) -> None:
        if self.step_count == 0:
            self.begin_step()
        unit, j = self._unit_of[id(p)]
        off = unit.offsets[j]
        with torch.no_grad():
            self.grad_pool[off:off + p.numel()].view(p.shape).copy_(p.grad)
        p.grad = None
        if j not in unit.staged:
            unit.staged.add(j)
            unit.pending -= 1
        if unit.pending == 0:
            self._launch_ready()

    def _launch_ready(self) -> None:
        while self._next < len(self.order) and self.order[self._next].pending == 0:
            unit = self.order[self._next]
            self._next += 1
            if not unit.launched:
                unit.launched = True
                self._update(unit)

    def _blocks(self, unit: _Unit) -> int:
        """CTAs of a unit's update: few while backward GEMMs still run beside it, the whole GPU for
        the last unit of the step (the embedding), which nothing overlaps."""
        if unit is self.order[-1]:
            return max(self.max_blocks, 4 * torch.cuda.get_device_properties(self.device).multi_processor_count)
        return self.max_blocks

    @torch.no_grad()
    def _update(self, unit: _Unit) -> None:
        st = self.state[unit.index]
        lo = unit.start + self.rank * unit.shard
        if self.cuda:
            from ..ops import ext

            main = torch.cuda.current_stream(self.device)
            self.stream.wait_stream(main)
            with torch.cuda.stream(self.stream):
                ext().peer_update(self.peer_grad, self.peer_param, self.peer_flags, self.flags, unit.index,
                                  self.rank, 0, lo, st["master"], st.get("m"), st.get("v"),
                                  0 if self.algo == "adamw" else 1, self.lr, self.betas[0], self.betas[1], self.eps,
                                  self.weight_decay, self.step_count, self.grad_scale, None, self.nonfinite,
                                  self._blocks(unit), self._step_t, self._epoch_t)
            return
        span = slice(unit.start, unit.start + unit.shard * self.world)
        grad = self.grad_pool[span].float()
        if self.distributed and self.world > 1:
            dist.all_reduce(grad, group=self.group)
        g = grad[self.rank * unit.shard:(self.rank + 1) * unit.shard] * self.grad_scale
        master = st["master"]
        if self.algo == "sgd":
            master.add_(g, alpha=-self.lr)
        else:
            beta1, beta2 = self.betas
            master.mul_(1 - self.lr * self.weight_decay)
            m = st["m"].float().mul_(beta1).add_(g, alpha=1 - beta1)
            v = st["v"].float().mul_(beta2).addcmul_(g, g, value=1 - beta2)
            bc1 = 1 - beta1 ** self.step_count
            bc2 = 1 - beta2 ** self.step_count
            master.addcdiv_(m, (v.sqrt() / math.sqrt(bc2)).add_(self.eps), value=-self.lr / bc1)
            st["m"].copy_(m)
            st["v"].copy_(v)
        self.param_pool[lo:lo + unit.shard].copy_(master)
        if self.distributed and self.world > 1:
            chunks = list(self.param_pool[span].chunk(self.world))
            dist.all_gather(chunks, chunks[self.rank].clone(), group=self.group)

    # -- checkpoint ----------------------------------------------------------------------------
    def state_dict(self) -> dict:
        return {"step": self.step_count, "algo": self.algo, "lr": self.lr, "betas": self.betas, "eps": self.eps,
                "weight_decay": self.weight_decay, "world": self.world, "rank": self.rank,
                "state": [{k: v for k, v in st.items()} for st in self.state]}

    def load_state_dict(self, state: dict) -> None:
        if int(state["world"]) != self.world:
            raise ValueError("optimizer state was saved with a different world size")
        self.step_count = int(state["step"])
        if self._step_t is not None:  # the flag epoch keeps counting from this process's history
            self._step_t.fill_(self.step_count)
        with torch.no_grad():
            for st, saved in zip(self.state, state["state"]):
                for key, value in saved.items():
                    st[key].copy_(value)


def decoder_units(model: nn.Module, exclude: set[int]) -> list[list[nn.Parameter]]:
    """Units of a decoder LM: the embedding, one per decoder layer, and the final norm with the
    head (the order of the forward pass). Parameters whose id is in ``exclude`` (expert weights,
    placed by expert parallelism) are left out."""
    inner = model.model
    seen = set(exclude)

    def take(params):
        out = []
        for p in params:
            if id(p) not in seen:  # a tied head weight stays in the embedding's unit
                seen.add(id(p))
                out.append(p)
        return out

    units = [take(inner.embed_tokens.parameters())]
    for layer in inner.layers:
        units.append(take(layer.parameters()))
    units.append(take(list(inner.norm.parameters()) + list(model.lm_head.parameters())))
    return [u for u in units if u]


__all__ = ["PeerShardedOptimizer", "decoder_units", "plan_units"]
