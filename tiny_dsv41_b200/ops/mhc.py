"""mHC (manifold-constrained hyper-connection) mixing ops for 4 residual streams.

* ``sinkhorn(comb, iters, eps)``: softmax over the last axis + eps, then alternating column /
  row normalisation (``dsv41_train/models/dsv4/mhc.py:466-489`` torch path, K5/K6 in Triton).
* ``collapse(streams [.., 4, H], w [.., 4])`` = sum_j w_j * stream_j in fp32 (K7/K8).
* ``expand(value [.., H], residual [.., 4, H], post [.., 4], comb [.., 4, 4])`` =
  post_k * value + sum_j comb_jk * residual_j in fp32 (K9/K10).

CUDA tensors run the warp-per-token kernels of ``csrc/mhc.cu``; CPU tensors the PyTorch forms.
"""

from __future__ import annotations

import torch

from ._ext import ext, on_gpu


def sinkhorn_reference(comb: torch.Tensor, iterations: int, eps: float) -> torch.Tensor:
    comb = torch.softmax(comb.float(), dim=-1) + eps
    comb = comb / (comb.sum(dim=-2, keepdim=True) + eps)
    for _ in range(iterations - 1):
        comb = comb / (comb.sum(dim=-1, keepdim=True) + eps)
        comb = comb / (comb.sum(dim=-2, keepdim=True) + eps)
    return comb


def collapse_reference(streams: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
    return (weights.unsqueeze(-1) * streams.float()).sum(-2).to(streams.dtype)


def expand_reference(value, residual, post, comb):
    mixed = torch.einsum("...jk,...jd->...kd", comb.float(), residual.float())
    return (post.unsqueeze(-1) * value.float().unsqueeze(-2) + mixed).to(residual.dtype)


class _Sinkhorn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, comb, iterations, eps):
        shape = comb.shape
        flat = comb.reshape(-1, 16).float().contiguous()
        out = ext().mhc_sinkhorn_fwd(flat, iterations, float(eps))
        ctx.save_for_backward(flat)
        ctx.meta = (iterations, eps, shape)
        return out.view(shape)

    @staticmethod
    def backward(ctx, grad):
        (flat,) = ctx.saved_tensors
        iterations, eps, shape = ctx.meta
        g = ext().mhc_sinkhorn_bwd(flat, grad.reshape(-1, 16).float().contiguous(), iterations, float(eps))
        return g.view(shape), None, None


class _Collapse(torch.autograd.Function):
    @staticmethod
    def forward(ctx, streams, weights):
        lead = streams.shape[:-2]
        h = streams.shape[-1]
        s = streams.reshape(-1, 4, h).contiguous()
        w = weights.reshape(-1, 4).float().contiguous()
        ctx.save_for_backward(s, w)
        ctx.meta = (lead, h, weights.dtype)
        return ext().mhc_collapse_fwd(s, w).view(*lead, h)

    @staticmethod
    def backward(ctx, grad):
        s, w = ctx.saved_tensors
        lead, h, wdtype = ctx.meta
        ds, dw = ext().mhc_collapse_bwd(grad.reshape(-1, h).contiguous(), s, w)
        return ds.view(*lead, 4, h), dw.view(*lead, 4).to(wdtype)


class _Expand(torch.autograd.Function):
    @staticmethod
    def forward(ctx, value, residual, post, comb):
        lead = residual.shape[:-2]
        h = residual.shape[-1]
        v = value.reshape(-1, h).contiguous()
        r = residual.reshape(-1, 4, h).contiguous()
        p = post.reshape(-1, 4).float().contiguous()
        c = comb.reshape(-1, 16).float().contiguous()
        ctx.save_for_backward(v, r, p, c)
        ctx.meta = (lead, h, post.dtype, comb.dtype)
        return ext().mhc_expand_fwd(v, r, p, c).view(*lead, 4, h)

    @staticmethod
    def backward(ctx, grad):
        v, r, p, c = ctx.saved_tensors
        lead, h, pdtype, cdtype = ctx.meta
        dv, dr, dp, dc = ext().mhc_expand_bwd(grad.reshape(-1, 4, h).contiguous(), v, r, p, c)
        return dv.view(*lead, h), dr.view(*lead, 4, h), dp.view(*lead, 4).to(pdtype), dc.view(*lead, 4, 4).to(cdtype)


def _kernel_ok(*tensors) -> bool:
    return on_gpu(*tensors) and all(t.numel() > 0 for t in tensors)


def sinkhorn(comb: torch.Tensor, iterations: int, eps: float) -> torch.Tensor:
    if comb.shape[-2:] == (4, 4) and _kernel_ok(comb):
        return _Sinkhorn.apply(comb, iterations, eps)
    return sinkhorn_reference(comb, iterations, eps)


def collapse(streams: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
    if streams.shape[-2] == 4 and streams.dtype == torch.bfloat16 and streams.shape[-1] % 8 == 0 and _kernel_ok(streams):
        return _Collapse.apply(streams, weights)
    return collapse_reference(streams, weights)


def expand(value, residual, post, comb):
    if (residual.shape[-2] == 4 and residual.dtype == torch.bfloat16 and value.dtype == torch.bfloat16
            and residual.shape[-1] % 8 == 0 and _kernel_ok(residual)):
        return _Expand.apply(value, residual, post, comb)
    return expand_reference(value, residual, post, comb)
