"""MoE routers with a fused score / top-k / normalise kernel.

``route(logits, ...)`` returns int32 expert ids [T, k] (descending by biased score) and fp32
weights [T, k]; the weights are differentiable w.r.t. the logits. An optional
:class:`AuxGradient` adds the gradient of the load-balancing loss
``E * sum_e f_e * P_e`` (``dsv41_train/models/qwen/model.py:400-435``,
``dsv41_train/models/dsv4/model.py:573-600``) during the same backward kernel.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from ._ext import ext, on_gpu

SCORE_FUNCS = {"softmax": 0, "sigmoid": 1, "sqrtsoftplus": 2}


class AuxGradient:
    """Per-expert gradient of the auxiliary loss w.r.t. softmax(router logits).

    The forward pass records expert counts; once all layers ran, :meth:`finalize` turns them
    into ``coef * E * count_e / (L*T)^2`` which every router backward adds to its dlogits.
    """

    def __init__(self) -> None:
        self.vector: torch.Tensor | None = None
        self.token_scale: torch.Tensor | None = None

    def set(self, vector: torch.Tensor | None, token_scale: torch.Tensor | None = None) -> None:
        """``vector`` [E]; optional ``token_scale`` [T] (0 for masked tokens)."""
        self.vector = None if vector is None else vector.float().contiguous()
        self.token_scale = None if token_scale is None else token_scale.float().reshape(-1, 1)

    def softmax_gradient(self, logits: torch.Tensor) -> torch.Tensor:
        """d aux / d logits through softmax(logits), in fp32."""
        p = torch.softmax(logits.float(), dim=-1)
        extra = p * (self.vector - (p * self.vector).sum(-1, keepdim=True))
        if self.token_scale is not None:
            extra = extra * self.token_scale
        return extra


def _scores_reference(logits: torch.Tensor, func: str) -> torch.Tensor:
    if func == "softmax":
        return torch.softmax(logits.float(), dim=-1)
    if func == "sigmoid":
        return torch.sigmoid(logits.float())
    return torch.sqrt(F.softplus(logits.float()))


def route_reference(logits, bias, k, func, normalize, norm_eps, scale):
    scores = _scores_reference(logits, func)
    selection = scores if bias is None else scores + bias
    indices = selection.topk(k, dim=-1).indices
    weights = scores.gather(-1, indices)
    if normalize and k > 1:
        weights = weights / (weights.sum(-1, keepdim=True) + norm_eps)
    return indices.to(torch.int32), weights * scale


class _Route(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, bias, k, func, normalize, norm_eps, scale, aux):
        ids, weights, scores = ext().router_fwd(logits.contiguous(), bias, k, SCORE_FUNCS[func], normalize,
                                                float(norm_eps), float(scale))
        ctx.save_for_backward(logits, ids, scores)
        ctx.meta = (func, normalize, norm_eps, scale, aux)
        ctx.mark_non_differentiable(ids)
        return ids, weights

    @staticmethod
    def backward(ctx, _dids, dweights):
        logits, ids, scores = ctx.saved_tensors
        func, normalize, norm_eps, scale, aux = ctx.meta
        if dweights is None:
            dweights = torch.zeros(ids.shape, dtype=torch.float32, device=ids.device)
        fused = aux is not None and aux.vector is not None and aux.token_scale is None
        vector = aux.vector if fused else None
        dlogits = ext().router_bwd(dweights.float().contiguous(), ids, scores, logits.contiguous(), vector,
                                   SCORE_FUNCS[func], normalize, float(norm_eps), float(scale))
        if aux is not None and aux.vector is not None and not fused:
            dlogits = (dlogits.float() + aux.softmax_gradient(logits)).to(dlogits.dtype)
        return dlogits, None, None, None, None, None, None, None


class _AuxHook(torch.autograd.Function):
    """CPU path: adds the auxiliary gradient through softmax(logits) explicitly."""

    @staticmethod
    def forward(ctx, logits, aux):
        ctx.save_for_backward(logits)
        ctx.aux = aux
        return logits.view_as(logits)

    @staticmethod
    def backward(ctx, grad):
        (logits,) = ctx.saved_tensors
        if ctx.aux.vector is None:
            return grad, None
        return grad + ctx.aux.softmax_gradient(logits).to(grad.dtype), None


def route(
    logits: torch.Tensor,
    k: int,
    *,
    func: str = "softmax",
    bias: torch.Tensor | None = None,
    normalize: bool = True,
    norm_eps: float = 0.0,
    scale: float = 1.0,
    aux: AuxGradient | None = None,
):
    if on_gpu(logits):
        return _Route.apply(logits, bias, k, func, normalize, norm_eps, scale, aux)
    if aux is not None and logits.requires_grad:
        logits = _AuxHook.apply(logits, aux)
    return route_reference(logits, bias, k, func, normalize, norm_eps, scale)
