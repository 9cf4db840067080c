"""Expert-major token movement and expert activations.

The routing metadata is built on the device without any host synchronisation (the reference
pulls split sizes to the host on every layer, ``dsv41_train/dispatch.py:87-89``): each expert's
routed rows form a segment starting at a multiple of ``BLOCK`` rows; padding rows are zero so
the grouped GEMMs (``ops.gemm.grouped_linear``) never need masks. Buffers have the static
capacity ``n_routes + E*(BLOCK-1)``; the number of rows actually used is a device scalar
(``Routing.total``) that the row-wise kernels read to skip the unused tail.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from ._ext import ext, on_gpu

BLOCK = 128


@dataclass
class Routing:
    route_rows: torch.Tensor   # [N, k] int32 row of each (item, slot) in the expert-major buffer (-1 = none)
    src: torch.Tensor          # [R_cap] int32 source item of each row (-1 = padding)
    offsets: torch.Tensor      # [E] int32 segment start rows
    rows: torch.Tensor         # [E] int32 segment sizes (multiples of BLOCK)
    counts: torch.Tensor       # [E] int64 routed rows per expert
    total: torch.Tensor        # [1] int32 rows in use (sum of segment sizes)
    capacity: int


def build_routing(ids: torch.Tensor, num_experts: int, block: int = BLOCK, *, slab_counts=None,
                  slab: int = 1) -> Routing:
    """Expert-major layout for ids [N, k] (entries < 0 are not routed).

    With ``slab_counts``, items are grouped in slabs of ``slab`` rows and only the first
    ``slab_counts[s]`` items of slab ``s`` are routed (the rest count as unrouted).
    """
    items, k = ids.shape
    if ids.is_cuda:
        route_rows, src, offsets, rows, counts, total = ext().moe_route_plan(
            ids.to(torch.int32).contiguous(), num_experts, block, slab_counts, slab)
        return Routing(route_rows, src, offsets, rows, counts, total, src.shape[0])
    if slab_counts is not None:
        live = (torch.arange(items, device=ids.device) % slab) < slab_counts.to(ids.device).repeat_interleave(slab)
        ids = torch.where(live.unsqueeze(1), ids, torch.full_like(ids, -1))
    flat = ids.reshape(-1).long()
    n = flat.numel()
    valid = flat >= 0
    keyed = torch.where(valid, flat, torch.full_like(flat, num_experts))
    counts_all = torch.bincount(keyed, minlength=num_experts + 1)
    counts = counts_all[:num_experts]
    padded = (counts + block - 1) // block * block
    seg_off = torch.cumsum(padded, 0) - padded
    start = torch.cumsum(counts_all, 0) - counts_all
    order = torch.argsort(keyed, stable=True)
    sorted_e = keyed[order]
    rank_in = torch.arange(n, device=ids.device) - start[sorted_e]
    seg_off_ext = torch.cat((seg_off, seg_off.new_zeros(1)))
    dest = torch.where(sorted_e < num_experts, seg_off_ext[sorted_e] + rank_in, torch.full_like(rank_in, -1))
    route_rows = torch.empty(n, dtype=torch.long, device=ids.device)
    route_rows[order] = dest
    capacity = (n + num_experts * (block - 1) + block - 1) // block * block
    src = torch.full((capacity + 1,), -1, dtype=torch.int32, device=ids.device)
    # invalid routes write into the spare last slot, which is then dropped
    src[torch.where(dest >= 0, dest, torch.full_like(dest, capacity))] = torch.div(order, k, rounding_mode="floor").to(torch.int32)
    src = src[:capacity]
    total = padded.sum().to(torch.int32).reshape(1)
    return Routing(route_rows.view(items, k).to(torch.int32), src.contiguous(), seg_off.to(torch.int32),
                   padded.to(torch.int32), counts, total, capacity)


class _Gather(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, src, route_rows, total):
        ctx.save_for_backward(route_rows)
        return ext().moe_gather(x.contiguous(), src, total)

    @staticmethod
    def backward(ctx, drows):
        (route_rows,) = ctx.saved_tensors
        return ext().moe_combine(drows.contiguous(), route_rows, None), None, None, None


class _Combine(torch.autograd.Function):
    @staticmethod
    def forward(ctx, rows, route_rows, weights, src, total):
        ctx.save_for_backward(rows, route_rows, weights, src, total)
        return ext().moe_combine(rows.contiguous(), route_rows, weights)

    @staticmethod
    def backward(ctx, dout):
        rows, route_rows, weights, src, total = ctx.saved_tensors
        need_dw = weights is not None and ctx.needs_input_grad[2]
        drows, dw = ext().moe_combine_bwd(dout.contiguous(), rows, route_rows, weights, need_dw)
        ext().moe_zero_padding(drows, src, total)
        return drows, None, (dw if need_dw else None), None, None


def gather(x: torch.Tensor, routing: Routing) -> torch.Tensor:
    """[N, H] -> expert-major [R_cap, H] (padding rows zero)."""
    if on_gpu(x):
        return _Gather.apply(x, routing.src, routing.route_rows, routing.total)
    out = x.new_zeros(routing.capacity, x.shape[-1])
    valid = routing.src >= 0
    out[valid] = x[routing.src[valid].long()]
    return out


def combine(rows: torch.Tensor, routing: Routing, weights: torch.Tensor | None) -> torch.Tensor:
    """sum_slot weights[t, slot] * rows[route_rows[t, slot]] in fp32, fixed slot order."""
    if on_gpu(rows):
        return _Combine.apply(rows, routing.route_rows, None if weights is None else weights.float().contiguous(),
                              routing.src, routing.total)
    index = routing.route_rows.long()
    picked = rows[index.clamp_min(0)].float() * (index >= 0).unsqueeze(-1)
    if weights is not None:
        picked = picked * weights.float().unsqueeze(-1)
    return picked.sum(1).to(rows.dtype)


def swiglu_reference(gate_up, weights=None, interleaved=False, limit=0.0):
    if interleaved:
        gate, up = gate_up.unflatten(-1, (-1, 2)).unbind(-1)
    else:
        gate, up = gate_up.chunk(2, dim=-1)
    gate, up = gate.float(), up.float()
    if limit > 0:
        gate = gate.clamp(max=limit)
        up = up.clamp(-limit, limit)
    silu = F.silu(gate)
    silu = torch.where(torch.isneginf(gate), torch.zeros_like(silu), silu)
    out = silu * up
    if weights is not None:
        out = out * weights.float().unsqueeze(-1)
    return out.to(gate_up.dtype)


class _SwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gate_up, weights, interleaved, limit, total):
        ctx.save_for_backward(gate_up, weights, total)
        ctx.meta = (interleaved, limit)
        return ext().swiglu_fwd(gate_up.contiguous(), weights, interleaved, float(limit), total)

    @staticmethod
    def backward(ctx, dout):
        gate_up, weights, total = ctx.saved_tensors
        interleaved, limit = ctx.meta
        need_dw = weights is not None and ctx.needs_input_grad[1]
        dgu, dw = ext().swiglu_bwd(dout.contiguous(), gate_up, weights, interleaved, float(limit), need_dw, total)
        return dgu, (dw if need_dw else None), None, None, None


def swiglu(gate_up: torch.Tensor, weights: torch.Tensor | None = None, *, interleaved: bool = False,
           limit: float = 0.0, total: torch.Tensor | None = None) -> torch.Tensor:
    """silu(gate) * up (optionally clamped, optionally times a per-row weight). ``total``: optional
    int32 device scalar; rows at or beyond it are skipped (left undefined)."""
    if on_gpu(gate_up):
        w = None if weights is None else weights.float().contiguous()
        return _SwiGLU.apply(gate_up, w, interleaved, limit, total)
    return swiglu_reference(gate_up, weights, interleaved, limit)
