"""Expert-parallel dispatch/combine over NVLink peer memory (fused path 1, transfer half).

Replaces the NCCL all-to-alls of ``dsv41_train/dispatch.py`` / ``models/dsv4/moe/dispatch.py``:

* symmetric buffers per rank (``torch.distributed._symmetric_memory``), peers' base addresses
  are handed to the kernels of ``csrc/ep_nvlink.cu``, which store directly into peer HBM;
* each token crosses NVLink once per destination rank (dedupe over its top-k experts) and the
  combine returns one pre-reduced row per (token, destination) - fewer bytes than the reference;
* routing metadata never leaves the device: no split sizes are pulled to the host, the
  receive layout is a fixed slab per source and the rows in use are device scalars;
* ready/free epoch flags with release/acquire ordering and bounded polls (status word on timeout).

The received rows are permuted into the 128-row aligned expert-major layout consumed by the
tcgen05 grouped GEMMs.
"""

from __future__ import annotations

import os

import torch
import torch.distributed as dist

from .. import ops
from ..ops import moe as moe_ops
from ..utils.trace import nvtx_range
from . import replay
from .dispatch import DispatchBatch, TokenDispatcher

# rows of the flag buffer
_RECV_READY, _RECV_FREE, _RET_READY, _RET_FREE, _COUNTS = range(5)
_CANARY = 0x5A5A  # int16 pattern of the debug guard rows


class _Workspace:
    """Symmetric buffers and peer pointer tables, shared by all MoE layers of one dispatcher."""

    def __init__(self, group, ep: int, rank: int, t_cap: int, hidden: int, k: int, device) -> None:
        import torch.distributed._symmetric_memory as symm

        self.ep, self.rank, self.t_cap, self.hidden, self.k = ep, rank, t_cap, hidden, k
        self.device = device
        # debug mode TDSV_EP_CANARY=1: one guard row after each row slab, filled with a pattern that
        # check_canaries() verifies after every exchange (an out-of-range peer write lands there)
        self.canary = os.environ.get("TDSV_EP_CANARY", "") not in ("", "0")
        guard = 1 if self.canary else 0
        recv = symm.empty(ep * t_cap + guard, hidden, dtype=torch.bfloat16, device=device)
        ret = symm.empty(ep * t_cap + guard, hidden, dtype=torch.bfloat16, device=device)
        self.recv = recv[:ep * t_cap].view(ep, t_cap, hidden)
        self.ret = ret[:ep * t_cap].view(ep, t_cap, hidden)
        self._guards = {"recv": recv[ep * t_cap:].view(torch.int16), "ret": ret[ep * t_cap:].view(torch.int16)}
        for g in self._guards.values():
            g.fill_(_CANARY)
        self._slabs = {"recv": recv, "ret": ret}
        self.meta = symm.empty(ep, t_cap, 2 * k, dtype=torch.int32, device=device)
        self.retw = symm.empty(ep, t_cap, k, dtype=torch.float32, device=device)
        self.flags = symm.empty(5, ep, dtype=torch.int32, device=device)
        self.flags.zero_()
        handles = {}
        for name in ("recv", "ret", "meta", "retw", "flags"):
            handles[name] = symm.rendezvous(self._slabs.get(name, getattr(self, name)), group)
        torch.cuda.synchronize(device)
        dist.barrier(group=group)

        def table(name, offset=0):
            ptrs = [int(p) + offset for p in handles[name].buffer_ptrs]
            return torch.tensor(ptrs, dtype=torch.int64, device=device)

        self.peer_recv = table("recv")
        self.peer_ret = table("ret")
        self.peer_meta = table("meta")
        self.peer_retw = table("retw")
        self.peer_flags = [table("flags", row * ep * 4) for row in range(5)]
        self.done = torch.zeros(2, dtype=torch.int32, device=device)
        # Epoch of an exchange = device base + host offset. The offsets count this step's exchanges
        # and the bases advance on the stream at end_step(), so a CUDA graph captured over a step
        # replays with fresh epochs. Without end_step() calls the bases stay 0 and the offsets
        # are plain running epochs.
        self.epoch_base = torch.zeros(2, dtype=torch.int32, device=device)  # [recv, ret]
        self.recv_epoch = 0
        self.ret_epoch = 0
        self.any_recv = False  # a slab was filled before: wait for its release before the next push
        self.any_ret = False
        self._handles = handles

    def flag_row(self, row: int) -> torch.Tensor:
        return self.flags[row]

    def recv_base(self) -> torch.Tensor:
        return self.epoch_base[0:1]

    def ret_base(self) -> torch.Tensor:
        return self.epoch_base[1:2]

    def end_step(self) -> None:
        """Fold this step's exchanges into the device bases (one small kernel, stream-ordered)."""
        # scalar adds: the amounts are kernel arguments, so a captured graph replays them as they are
        if self.recv_epoch:
            self.epoch_base[0:1].add_(self.recv_epoch)
        if self.ret_epoch:
            self.epoch_base[1:2].add_(self.ret_epoch)
        self.recv_epoch = 0
        self.ret_epoch = 0

    def check_canaries(self, where: str) -> None:
        """Debug mode only (synchronises): raise if a guard row after a slab was overwritten."""
        if not self.canary:
            return
        for name, guard in self._guards.items():
            if not bool((guard == _CANARY).all()):
                raise RuntimeError(f"NVLink EP: the guard row after the {name} slab was overwritten ({where}); "
                                   "a peer wrote outside its slab")


class _Exchange:
    """Routing state of one MoE call, shared between its dispatch and combine autograd nodes."""

    def __init__(self, ws: _Workspace, tokens: int, e_local: int) -> None:
        self.ws = ws
        self.tokens = tokens
        self.e_local = e_local
        self.dest_mask = None
        self.slot = None
        self.counts = None
        self.recv_counts = None
        self.routing = None
        self.local_w = None
        self.owner = None
        self.recording = False  # activation-checkpoint replay (see parallel.replay)
        self.replaying = False
        self.cached_recv = None
        self.cached_out = None

    # -- transfer primitives --------------------------------------------------------------
    def push_to_receivers(self, rows: torch.Tensor, ids=None, weights=None) -> None:
        """rows [T, H] -> every destination's recv slab (waits until the slab is free)."""
        ws, C = self.ws, ops.ext()
        if ws.any_recv:  # the previous contents of the peers' slabs were released
            C.ep_wait(ws.flag_row(_RECV_FREE), ws.recv_epoch, ws.recv_base())
        ws.any_recv = True
        ws.recv_epoch += 1
        with_meta = ids is not None
        C.ep_push_rows(rows.contiguous(), self.dest_mask, self.slot, ws.peer_recv,
                       ws.peer_meta if with_meta else None, ids, weights, ws.t_cap, self.e_local, ws.done[0:1],
                       ws.peer_flags[_RECV_READY], ws.peer_flags[_COUNTS] if with_meta else None,
                       self.counts if with_meta else None, ws.rank, ws.recv_epoch, ws.recv_base())
        C.ep_wait(ws.flag_row(_RECV_READY), ws.recv_epoch, ws.recv_base())
        ws.check_canaries("dispatch")

    def release_recv(self) -> None:
        ws = self.ws
        ops.ext().ep_signal(ws.peer_flags[_RECV_FREE], None, None, ws.rank, ws.recv_epoch, ws.recv_base())

    def push_to_sources(self, y: torch.Tensor, route: torch.Tensor, weights=None, extra=None) -> None:
        """Per received row: sum_j w_j * y[route[row, j]] -> the source's ret slab (+ extra floats)."""
        ws, C = self.ws, ops.ext()
        if ws.any_ret:
            C.ep_wait(ws.flag_row(_RET_FREE), ws.ret_epoch, ws.ret_base())
        ws.any_ret = True
        ws.ret_epoch += 1
        C.ep_combine_push(y.contiguous(), route, weights, self.recv_counts, ws.peer_ret, extra,
                          ws.peer_retw if extra is not None else None, ws.t_cap, ws.done[1:2],
                          ws.peer_flags[_RET_READY], ws.rank, ws.ret_epoch, ws.ret_base())
        C.ep_wait(ws.flag_row(_RET_READY), ws.ret_epoch, ws.ret_base())
        ws.check_canaries("combine")

    def release_ret(self) -> None:
        ws = self.ws
        ops.ext().ep_signal(ws.peer_flags[_RET_FREE], None, None, ws.rank, ws.ret_epoch, ws.ret_base())


class _Dispatch(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weights, ids, ex: _Exchange):
        ws = ex.ws
        t, k = ids.shape
        ids32 = ids.to(torch.int32).contiguous()
        ex.owner = torch.div(ids.long(), ex.e_local, rounding_mode="floor")
        ex.dest_mask, ex.slot, ex.counts = ops.ext().ep_dest_plan(ids32, ex.e_local, ws.ep)
        ex.push_to_receivers(x, ids32, weights.float().contiguous())
        ex.recv_counts = ws.flag_row(_COUNTS).clone()
        meta = ws.meta.view(ws.ep * ws.t_cap, 2 * k)
        live = (torch.arange(ws.t_cap, device=x.device).unsqueeze(0) < ex.recv_counts.unsqueeze(1)).reshape(-1, 1)
        local_w = torch.where(live, meta[:, k:].view(torch.float32), torch.zeros_like(meta[:, k:].view(torch.float32)))
        # rows past each source's live count are masked inside the routing plan
        ex.routing = moe_ops.build_routing(meta[:, :k].contiguous(), ex.e_local, slab_counts=ex.recv_counts,
                                           slab=ws.t_cap)
        received = ws.recv.view(ws.ep * ws.t_cap, ws.hidden)
        rows = ops.ext().moe_gather(received, ex.routing.src, ex.routing.total)
        if ex.recording:  # the receive slabs, not the capacity-sized expert-major buffer (~8x smaller)
            ex.cached_recv = received.clone()
        ex.release_recv()
        ex.local_w = local_w.contiguous()
        ctx.ex = ex
        return rows, ex.local_w.clone()

    @staticmethod
    def backward(ctx, d_rows, d_local_w):
        ex = ctx.ex
        ws = ex.ws
        k = ex.routing.route_rows.shape[1]
        extra = None if d_local_w is None else d_local_w.float().contiguous()
        # per received row: sum over its local expert rows, pushed back to the source (+ weight grads)
        ex.push_to_sources(d_rows, ex.routing.route_rows, None, extra)
        dx = ops.ext().ep_reduce_returned(ws.ret, ex.dest_mask, ex.slot, ex.tokens)
        dweights = None
        if extra is not None:
            retw = ws.retw  # [ep, t_cap, k]
            gathered = retw[ex.owner, ex.slot.long().gather(1, ex.owner)]  # [T, k, k]
            dweights = torch.diagonal(gathered, dim1=1, dim2=2).contiguous()
        ex.release_ret()
        return dx, dweights, None, None


class _Combine(torch.autograd.Function):
    @staticmethod
    def forward(ctx, y, local_w, ex: _Exchange):
        ws = ex.ws
        ex.push_to_sources(y, ex.routing.route_rows, local_w)
        out = ops.ext().ep_reduce_returned(ws.ret, ex.dest_mask, ex.slot, ex.tokens)
        ex.release_ret()
        ctx.ex = ex
        ctx.save_for_backward(y, local_w)
        return out

    @staticmethod
    def backward(ctx, dout):
        ex = ctx.ex
        ws = ex.ws
        y, local_w = ctx.saved_tensors
        ex.push_to_receivers(dout)
        drecv = ws.recv.view(ws.ep * ws.t_cap, ws.hidden)
        need_w = local_w is not None and ctx.needs_input_grad[1]
        dy, dw = ops.ext().moe_combine_bwd(drecv, y, ex.routing.route_rows, local_w, need_w)
        ops.ext().moe_zero_padding(dy, ex.routing.src, ex.routing.total)
        ex.release_recv()
        return dy, (dw if need_w else None), None


class _ScatterRowWeights(torch.autograd.Function):
    @staticmethod
    def forward(ctx, local_w, route_rows, capacity):
        ctx.save_for_backward(route_rows)
        out = torch.zeros(capacity + 1, dtype=torch.float32, device=local_w.device)
        idx = route_rows.reshape(-1).long()
        out[torch.where(idx >= 0, idx, torch.full_like(idx, capacity))] = local_w.reshape(-1)
        return out[:capacity]

    @staticmethod
    def backward(ctx, grad):
        (route_rows,) = ctx.saved_tensors
        idx = route_rows.long()
        g = torch.cat((grad, grad.new_zeros(1)))
        return g[torch.where(idx >= 0, idx, torch.full_like(idx, grad.shape[0]))], None, None


class _ReplayDispatch(_Dispatch):
    """Recompute of a recorded dispatch: the recorded rows, no transfer; same backward."""

    @staticmethod
    def forward(ctx, x, weights, ids, ex: _Exchange):
        if ex.cached_recv is None:
            raise RuntimeError("the recorded dispatch was already replayed once")
        ctx.ex = ex
        rows = ops.ext().moe_gather(ex.cached_recv, ex.routing.src, ex.routing.total)
        ex.cached_recv = None  # the backward needs only the routing state
        return rows, ex.local_w.clone()


class _ReplayCombine(_Combine):
    """Recompute of a recorded combine: the recorded output, no transfer; same backward."""

    @staticmethod
    def forward(ctx, y, local_w, ex: _Exchange):
        if ex.cached_out is None:
            raise RuntimeError("the recorded combine was already replayed once")
        ctx.ex = ex
        ctx.save_for_backward(y, local_w)
        # A fresh output tensor: returning the recorded one would give it this node as grad_fn,
        # and the record (held by the checkpoint frame) would then keep the frame alive.
        out, ex.cached_out = ex.cached_out.clone(), None
        return out


class NVLinkTokenDispatcher(TokenDispatcher):
    """EP dispatcher whose transfers are this repository's peer-memory kernels."""

    def __init__(self, mesh, max_tokens: int = 8192) -> None:
        super().__init__()
        if mesh.ndim != 1:
            raise ValueError("the EP mesh must be one-dimensional")
        self.mesh = mesh
        self.size = mesh.size()
        self.rank = mesh.get_local_rank()
        self.group = mesh.get_group()
        self.max_tokens = max_tokens
        self._ws: _Workspace | None = None

    def expert_range(self, num_experts: int) -> tuple[int, int]:
        if num_experts % self.size:
            raise ValueError(f"num_experts ({num_experts}) must divide EP size ({self.size})")
        self.num_experts = num_experts
        local = num_experts // self.size
        return self.rank * local, (self.rank + 1) * local

    def end_step(self) -> None:
        """Advance the device-side exchange epochs past this step (see ``_Workspace.end_step``)."""
        if self._ws is not None:
            self._ws.end_step()

    def abort_step(self) -> None:
        """Drop the offsets counted by a step that never ran (a failed CUDA-graph capture)."""
        if self._ws is not None:
            self._ws.recv_epoch = self._ws.ret_epoch = 0

    def _workspace(self, tokens: int, hidden: int, k: int, device) -> _Workspace:
        ws = self._ws
        if ws is None or ws.t_cap < tokens or ws.hidden != hidden or ws.k != k:
            cap = max(tokens, self.max_tokens)
            self._ws = ws = _Workspace(self.group, self.size, self.rank, cap, hidden, k, device)
        return ws

    def dispatch(self, x, ids, weights) -> DispatchBatch:
        if self.num_experts is None:
            raise RuntimeError("attach the dispatcher to an expert module before use")
        if not x.is_cuda:
            raise RuntimeError("the NVLink dispatcher needs CUDA tensors")
        handle, mode = replay.current()
        with nvtx_range("ep.dispatch"):
            if mode == "replay":
                ex = handle.next()
                rows, local_w = _ReplayDispatch.apply(x, weights, ids, ex)
            else:
                ws = self._workspace(x.shape[0], x.shape[1], ids.shape[1], x.device)
                ex = _Exchange(ws, x.shape[0], self.num_experts // self.size)
                ex.recording = mode == "record"
                rows, local_w = _Dispatch.apply(x, weights, ids, ex)
                if ex.recording:
                    handle.record(ex)
        ex.replaying = mode == "replay"
        routing = ex.routing
        return DispatchBatch(rows, routing.offsets, routing.rows, None,
                             {"exchange": ex, "local_w": local_w, "routing": routing}, routing.total)

    def row_weights(self, batch: DispatchBatch) -> torch.Tensor:
        routing = batch.state["routing"]
        return _ScatterRowWeights.apply(batch.state["local_w"], routing.route_rows, routing.capacity)

    def combine(self, y, batch: DispatchBatch, *, weighted: bool = True):
        ex = batch.state["exchange"]
        local_w = batch.state["local_w"] if weighted else None
        if ex.replaying:
            return _ReplayCombine.apply(y, local_w, ex)
        with nvtx_range("ep.combine"):
            out = _Combine.apply(y, local_w, ex)
        if ex.recording:
            ex.cached_out = out.detach()
        return out


__all__ = ["NVLinkTokenDispatcher"]
