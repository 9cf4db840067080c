"""bf16 GEMMs on the persistent tcgen05 kernel (``csrc/gemm_tc.cu``).

* :func:`linear` - ``y = x @ w.T`` with w in ``nn.Linear`` layout; backward uses the MN-major
  operand forms (dx = dy @ w, dw = dy^T @ x) so no transposed copies are made.
* :func:`grouped_linear` - expert-major grouped GEMM over 128-row aligned expert segments whose
  offsets/sizes are device tensors (replaces ``torch._grouped_mm`` in
  ``dsv41_train/models/dsv4/moe/module.py:78-99`` and the per-expert loop of
  ``dsv41_train/models/qwen/model.py:231-238``).
"""

from __future__ import annotations

import torch

from ._ext import ext, on_gpu


def _kernel_ok(*tensors: torch.Tensor) -> bool:
    return all(t.dtype == torch.bfloat16 for t in tensors)


def matmul_nt(a: torch.Tensor, b: torch.Tensor, out_dtype=torch.bfloat16) -> torch.Tensor:
    """a [M, K] @ b[N, K]^T on the tensor-core kernel."""
    out = torch.empty(a.shape[0], b.shape[0], dtype=out_dtype, device=a.device)
    ext().gemm(a.contiguous(), b.contiguous(), out, False, False, False)
    return out


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, replayable=False):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous()
        handle, mode = (None, None)
        if replayable:
            from ..parallel import replay

            handle, mode = replay.current()
        if mode == "replay":  # checkpoint recompute: the first pass's product of the same operands
            out = handle.next_attention().clone()
        else:
            out = torch.empty(x2.shape[0], weight.shape[0], dtype=torch.bfloat16, device=x.device)
            ext().gemm(x2, weight, out, False, False, False)
            if mode == "record":
                handle.record_attention(out.detach())
        ctx.save_for_backward(x2, weight)
        ctx.shape = shape
        return out.view(*shape[:-1], weight.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2, weight = ctx.saved_tensors
        dy2 = dy.reshape(-1, weight.shape[0]).contiguous()
        dx = dw = None
        if ctx.needs_input_grad[0]:
            dx = torch.empty_like(x2)
            ext().gemm(dy2, weight, dx, False, True, False)
            dx = dx.view(ctx.shape)
        if ctx.needs_input_grad[1]:
            dw = torch.empty_like(weight)
            ext().gemm(dy2, x2, dw, True, True, False)
        return dx, dw, None


def linear(x: torch.Tensor, weight: torch.Tensor, *, replayable: bool = False) -> torch.Tensor:
    """``x @ weight.T``. ``replayable``: under activation checkpointing the recompute reuses the
    first pass's product (kept by ``parallel/replay.py``) instead of running the GEMM again - for
    small outputs whose recompute costs more than the memory to keep them."""
    if on_gpu(x) and _kernel_ok(x, weight) and weight.shape[0] % 8 == 0 and weight.shape[1] % 8 == 0:
        return _Linear.apply(x, weight, replayable)
    return torch.nn.functional.linear(x, weight.to(x.dtype))


def grouped_linear_reference(x, weight, offsets, rows):
    """Plain PyTorch restatement. Every group contributes a (possibly empty) product, so the result
    always depends on ``x`` and ``weight`` in autograd, even when no rows are routed: a rank whose
    experts received nothing must still run the same backward collectives as its peers."""
    pieces, at = [], 0
    for g, (start, count) in sorted(enumerate(zip(offsets.tolist(), rows.tolist())), key=lambda item: item[1][0]):
        if start > at:
            pieces.append(x.new_zeros(start - at, weight.shape[1]))
        pieces.append((x[start:start + count].float() @ weight[g].float().t()).to(x.dtype))
        at = max(at, start + count)
    if at < x.shape[0]:
        pieces.append(x.new_zeros(x.shape[0] - at, weight.shape[1]))
    return torch.cat(pieces) if pieces else x.new_zeros(x.shape[0], weight.shape[1])


class _GroupedLinear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, offsets, rows):
        out = torch.empty(x.shape[0], weight.shape[1], dtype=torch.bfloat16, device=x.device)
        ext().grouped_gemm_m(x, weight, offsets, rows, out, False, x.shape[0])
        ctx.save_for_backward(x, weight, offsets, rows)
        return out

    @staticmethod
    def backward(ctx, dy):
        x, weight, offsets, rows = ctx.saved_tensors
        dy = dy.contiguous()
        dx = dw = None
        if ctx.needs_input_grad[0]:
            dx = torch.empty_like(x)
            ext().grouped_gemm_m(dy, weight, offsets, rows, dx, True, x.shape[0])
        if ctx.needs_input_grad[1]:
            dw = torch.empty_like(weight)
            ext().grouped_gemm_k(dy, x, offsets, rows, dw, False)
        return dx, dw, None, None


def grouped_linear(x: torch.Tensor, weight: torch.Tensor, offsets: torch.Tensor, rows: torch.Tensor) -> torch.Tensor:
    """Rows ``[offsets[g], offsets[g] + rows[g])`` of x times ``weight[g].T`` (weight [G, N, K]).

    Row segments must be 128-aligned with zero padding rows (see ops.moe.build_routing).
    """
    if on_gpu(x) and _kernel_ok(x, weight):
        return _GroupedLinear.apply(x.contiguous(), weight.contiguous(), offsets, rows)
    return grouped_linear_reference(x, weight, offsets, rows)
