"""Expert-major token movement and expert activations.

The routing metadata is built on the device without any host synchronisation (the reference
pulls split sizes to the host on every layer, ``dsv41_train/dispatch.py:87-89``): each expert's
routed rows form a segment starting at a multiple of ``BLOCK`` rows; padding rows are zero so
the grouped GEMMs (``ops.gemm.grouped_linear``) never need masks. The buffer capacity is the
static upper bound ``T*k + E*(BLOCK-1)``.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from ._ext import ext, on_gpu

BLOCK = 128


@dataclass
class Routing:
    route_rows: torch.Tensor   # [T, k] int32 row of each (token, slot) in the expert-major buffer
    src: torch.Tensor          # [R_cap] int32 source token of each row (-1 = padding)
    offsets: torch.Tensor      # [E] int32 segment start rows
    rows: torch.Tensor         # [E] int32 segment sizes (multiples of BLOCK)
    counts: torch.Tensor       # [E] int64 routed rows per expert
    capacity: int


def build_routing(ids: torch.Tensor, num_experts: int, block: int = BLOCK) -> Routing:
    tokens, k = ids.shape
    flat = ids.reshape(-1).long()
    n = flat.numel()
    counts = torch.bincount(flat, minlength=num_experts)
    padded = (counts + block - 1) // block * block
    seg_off = torch.cumsum(padded, 0) - padded
    start = torch.cumsum(counts, 0) - counts
    order = torch.argsort(flat, stable=True)
    sorted_e = flat[order]
    dest = seg_off[sorted_e] + (torch.arange(n, device=ids.device) - start[sorted_e])
    route_rows = torch.empty(n, dtype=torch.long, device=ids.device)
    route_rows[order] = dest
    capacity = n + num_experts * (block - 1)
    capacity = (capacity + block - 1) // block * block
    src = torch.full((capacity,), -1, dtype=torch.int32, device=ids.device)
    src[dest] = torch.div(order, k, rounding_mode="floor").to(torch.int32)
    return Routing(route_rows.view(tokens, k).to(torch.int32), src, seg_off.to(torch.int32),
                   padded.to(torch.int32), counts, capacity)


class _Gather(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, src, route_rows):
        ctx.save_for_backward(route_rows)
        return ext().moe_gather(x.contiguous(), src)

    @staticmethod
    def backward(ctx, drows):
        (route_rows,) = ctx.saved_tensors
        return ext().moe_combine(drows.contiguous(), route_rows, None), None, None


class _Combine(torch.autograd.Function):
    @staticmethod
    def forward(ctx, rows, route_rows, weights, src):
        ctx.save_for_backward(rows, route_rows, weights, src)
        return ext().moe_combine(rows.contiguous(), route_rows, weights)

    @staticmethod
    def backward(ctx, dout):
        rows, route_rows, weights, src = ctx.saved_tensors
        need_dw = weights is not None and ctx.needs_input_grad[2]
        drows, dw = ext().moe_combine_bwd(dout.contiguous(), rows, route_rows, weights, need_dw)
        ext().moe_zero_padding(drows, src)
        return drows, None, (dw if need_dw else None), None


def gather(x: torch.Tensor, routing: Routing) -> torch.Tensor:
    """[T, H] -> expert-major [R_cap, H] (padding rows zero)."""
    if on_gpu(x):
        return _Gather.apply(x, routing.src, routing.route_rows)
    out = x.new_zeros(routing.capacity, x.shape[-1])
    valid = routing.src >= 0
    out[valid] = x[routing.src[valid].long()]
    return out


def combine(rows: torch.Tensor, routing: Routing, weights: torch.Tensor | None) -> torch.Tensor:
    """sum_slot weights[t, slot] * rows[route_rows[t, slot]] in fp32, fixed slot order."""
    if on_gpu(rows):
        return _Combine.apply(rows, routing.route_rows, None if weights is None else weights.float().contiguous(),
                              routing.src)
    picked = rows[routing.route_rows.long()].float()
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
    def forward(ctx, gate_up, weights, interleaved, limit):
        ctx.save_for_backward(gate_up, weights)
        ctx.meta = (interleaved, limit)
        return ext().swiglu_fwd(gate_up.contiguous(), weights, interleaved, float(limit))

    @staticmethod
    def backward(ctx, dout):
        gate_up, weights = ctx.saved_tensors
        interleaved, limit = ctx.meta
        need_dw = weights is not None and ctx.needs_input_grad[1]
        dgu, dw = ext().swiglu_bwd(dout.contiguous(), gate_up, weights, interleaved, float(limit), need_dw)
        return dgu, (dw if need_dw else None), None, None


def swiglu(gate_up: torch.Tensor, weights: torch.Tensor | None = None, *, interleaved: bool = False,
           limit: float = 0.0) -> torch.Tensor:
    """silu(gate) * up (optionally clamped, optionally times a per-row weight)."""
    if on_gpu(gate_up):
        w = None if weights is None else weights.float().contiguous()
        return _SwiGLU.apply(gate_up, w, interleaved, limit)
    return swiglu_reference(gate_up, weights, interleaved, limit)
