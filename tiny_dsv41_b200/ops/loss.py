"""Chunked LM-head cross entropy and selected-token log-probabilities.

:func:`linear_cross_entropy` never materialises the full ``[tokens, vocab]`` logits: for each
chunk of rows it runs the LM-head GEMM, the fused CE kernel (loss + in-place gradient), and the
two backward GEMMs, keeping only ``dX`` and an fp32 ``dW`` accumulator for autograd. It is the
sum-reduced CE of ``dsv41_train/models/dsv4/model.py:670-677`` / ``qwen/model.py:494-517``.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from ._ext import ext, on_gpu

IGNORE_INDEX = -100


class _LinearCrossEntropy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden, weight, targets, chunk):
        C = ext()
        rows = hidden.shape[0]
        vocab = weight.shape[0]
        need_dx = ctx.needs_input_grad[0]
        need_dw = ctx.needs_input_grad[1]
        if chunk >= rows:
            # one pass: logits -> in-place CE gradient -> dX and dW GEMMs (bf16 dW, K = all rows)
            logits = torch.empty(rows, vocab, dtype=torch.bfloat16, device=hidden.device)
            C.gemm(hidden, weight, logits, False, False, False)
            loss, _ = C.cross_entropy_fused(logits, targets, 1.0, IGNORE_INDEX, need_dx or need_dw)
            dx = dw = None
            if need_dx:
                dx = torch.empty_like(hidden)
                C.gemm(logits, weight, dx, False, True, False)
            if need_dw:
                dw = torch.empty_like(weight)
                C.gemm(logits, hidden, dw, True, True, False)
            ctx.save_for_backward(dx, dw)
            ctx.weight_dtype = weight.dtype
            return loss.sum()
        total = torch.zeros((), dtype=torch.float32, device=hidden.device)
        dx = torch.empty_like(hidden) if need_dx else None
        dw = torch.zeros(weight.shape, dtype=torch.float32, device=hidden.device) if need_dw else None
        for start in range(0, rows, chunk):
            stop = min(rows, start + chunk)
            h = hidden[start:stop]
            logits = torch.empty(stop - start, vocab, dtype=torch.bfloat16, device=hidden.device)
            C.gemm(h, weight, logits, False, False, False)
            loss, _ = C.cross_entropy_fused(logits, targets[start:stop], 1.0, IGNORE_INDEX, need_dx or need_dw)
            total += loss.sum()
            if need_dx:
                C.gemm(logits, weight, dx[start:stop], False, True, False)
            if need_dw:
                C.gemm(logits, h, dw, True, True, True)
        ctx.save_for_backward(dx, dw)
        ctx.weight_dtype = weight.dtype
        return total

    @staticmethod
    def backward(ctx, grad):
        dx, dw = ctx.saved_tensors
        gdx = None if dx is None else dx.mul_(grad.to(dx.dtype)) if dx.dtype == torch.float32 else (
            dx.float() * grad).to(dx.dtype)
        if dw is None:
            gdw = None
        elif dw.dtype == torch.float32:
            gdw = (dw * grad).to(ctx.weight_dtype)
        else:
            gdw = dw.mul_(grad.to(dw.dtype))
        return gdx, gdw, None, None


def linear_cross_entropy(hidden: torch.Tensor, weight: torch.Tensor, targets: torch.Tensor,
                         chunk: int | None = None) -> torch.Tensor:
    """Sum over rows of CE(hidden @ weight.T, targets) (rows with target -100 are ignored).

    ``chunk`` rows per pass; by default all rows at once when their bf16 logits fit in 4 GiB."""
    if chunk is None:
        chunk = hidden.numel() // hidden.shape[-1]
        if chunk * weight.shape[0] * 2 > 4 * 2 ** 30:
            chunk = max(128, (4 * 2 ** 30) // (weight.shape[0] * 2) // 128 * 128)
    hidden = hidden.reshape(-1, hidden.shape[-1])
    targets = targets.reshape(-1)
    if on_gpu(hidden) and hidden.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16:
        return _LinearCrossEntropy.apply(hidden.contiguous(), weight.contiguous(), targets.contiguous(), chunk)
    logits = F.linear(hidden, weight.to(hidden.dtype)).float()
    return F.cross_entropy(logits, targets, ignore_index=IGNORE_INDEX, reduction="sum")


class _TokenLogProb(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, targets, temperature):
        logp, lse = ext().token_logprob_fwd(logits.contiguous(), targets.contiguous(), float(temperature))
        ctx.save_for_backward(logits, targets, lse)
        ctx.temperature = temperature
        return logp

    @staticmethod
    def backward(ctx, dlogp):
        logits, targets, lse = ctx.saved_tensors
        return ext().token_logprob_bwd(logits, targets, lse, dlogp.contiguous(), float(ctx.temperature)), None, None


def token_log_probs(logits: torch.Tensor, targets: torch.Tensor, temperature: float = 1.0) -> torch.Tensor:
    """log_softmax(logits / T)[target] per row, fp32."""
    if on_gpu(logits):
        return _TokenLogProb.apply(logits, targets, temperature)
    return F.log_softmax(logits.float() / temperature, dim=-1).gather(-1, targets.unsqueeze(-1)).squeeze(-1)
