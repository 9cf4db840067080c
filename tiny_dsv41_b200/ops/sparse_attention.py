"""DSV4 sparse attention (sliding window + selected compressed KV + per-head sink logit) and the
sparse-indexer scores.

``sparse_attention(q [B,H,L,D], kv [B,S,D], window_idx [B,L,W], window_mask [B,L,W],
compressed [B,C,D] | None, compressed_idx [B,L,K] | None, sinks [H])`` returns [B,L,H,D]; the
softmax runs over window logits, selected compressed logits and the sink logit together, and the
sink contributes no value (``dsv41_train/models/dsv4/attention/module.py:473-534`` and the Triton
K1/K2 kernels of ``sparse_attention.py``).

``index_scores`` = sum_h w[q,h] * relu(q_h . k) * d^-1/2 over each query's visible compressed
keys (``sparse_indexer.py:156-172``), -inf outside [start, end) or outside the candidate mask.

On CUDA, ``index_scores`` runs the tcgen05 kernel of ``csrc/index_scores.cu`` (keys as the M
operand, the block's (query, head) rows as N, relu / head weights / head reduction in the TMEM
epilogue; head dim 64 or 128, heads a power of two from 4 to 64). ``sparse_attention`` runs the
tcgen05 forward of ``csrc/sparse_attention.cu`` (gathered keys as the M operand, 64 heads as N,
online softmax seeded with the sink; bf16, head dim 128 / 256 / 512, no dropout) and its tcgen05
backward (dQ per token, dKV rows added with fp32 vector reductions, or with
``deterministic=True`` per-edge rows summed in a fixed order by an owner per KV row). Other shapes
run the restatement below, which is also the oracle on CPU.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from ._ext import ext, on_gpu


def _sparse_kernel_ok(query, kv, window_indices, compressed_kv, compressed_indices, dropout) -> bool:
    dim = query.shape[-1]
    return (dropout == 0.0 and query.dtype == torch.bfloat16 and kv.dtype == torch.bfloat16
            and dim in (128, 256, 512) and window_indices.shape[-1] + (
                0 if compressed_indices is None else compressed_indices.shape[-1]) > 0
            and (compressed_kv is None or compressed_kv.dtype == torch.bfloat16))


class _SparseAttention(torch.autograd.Function):
    """tcgen05 forward and backward (``csrc/sparse_attention.cu``). The backward adds the KV
    gradients of rows shared by several tokens with fp32 vector reductions; ``deterministic``
    stores every (token, entry) edge's KV gradient row instead and sums each KV row over its edges
    in ascending edge order, chunk by chunk (the ordered-dKV scheme of the reference's
    ``ordered_kv.py``), so repeated runs are bitwise equal."""

    @staticmethod
    def forward(ctx, query, kv, window_indices, window_mask, compressed_kv, compressed_indices, sinks, deterministic):
        q = query.transpose(1, 2).contiguous()  # [B, L, H, D]: free when the projection wrote it that way
        kv_c = kv.contiguous()
        widx = window_indices.long().contiguous()
        wmask = window_mask.bool().contiguous()
        comp = None if compressed_kv is None else compressed_kv.contiguous()
        cidx = None if compressed_indices is None else compressed_indices.long().contiguous()
        sk = sinks.float().contiguous()
        out, lse = ext().sparse_attention_fwd(q, kv_c, widx, wmask, comp, cidx, sk)
        ctx.deterministic = deterministic
        ctx.has_comp = comp is not None
        ctx.sinks_dtype = sinks.dtype
        ctx.save_for_backward(q, kv_c, widx, wmask, comp, cidx, sk, out, lse)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        q, kv, widx, wmask, comp, cidx, sinks, out, lse = ctx.saved_tensors
        chunk = None
        if ctx.deterministic:  # per-edge rows, each KV row summed by one owner in edge order
            batch, _, heads, dim = q.shape
            slots = widx.shape[-1] + (0 if cidx is None else cidx.shape[-1])
            per_token = batch * slots * ((heads + 63) // 64) * dim * 4
            chunk = max(1, _EDGE_BUFFER_BYTES // per_token)
        dq, dkv, dcomp, dsink = ext().sparse_attention_bwd(q, kv, widx, wmask, comp, cidx, sinks, out, lse,
                                                           grad_out.contiguous(), chunk)
        return (dq.transpose(1, 2), dkv.to(kv.dtype), None, None,
                dcomp.to(comp.dtype) if ctx.has_comp else None, None,
                dsink.sum(dim=(0, 1)).to(ctx.sinks_dtype), None)


_EDGE_BUFFER_BYTES = 512 * 2 ** 20  # per-chunk edge rows of the deterministic KV gradient


def sparse_attention(query, kv, window_indices, window_mask, compressed_kv, compressed_indices, sinks, *,
                     dropout: float = 0.0, deterministic: bool = False):
    if on_gpu(query) and _sparse_kernel_ok(query, kv, window_indices, compressed_kv, compressed_indices, dropout):
        return _SparseAttention.apply(query, kv, window_indices, window_mask, compressed_kv, compressed_indices,
                                      sinks, deterministic)
    return sparse_attention_reference(query, kv, window_indices, window_mask, compressed_kv, compressed_indices,
                                      sinks, dropout=dropout)


def sparse_attention_reference(query, kv, window_indices, window_mask, compressed_kv, compressed_indices, sinks, *,
                               dropout: float = 0.0):
    batch, heads, length, dim = query.shape
    rows = torch.arange(batch, device=query.device).view(-1, 1, 1)
    window_kv = kv[rows, window_indices.long()]  # [B, L, W, D]
    scale = dim ** -0.5
    logits = torch.einsum("bhld,blwd->bhlw", query, window_kv.to(query.dtype)) * scale
    logits = logits.masked_fill(~window_mask.unsqueeze(1), torch.finfo(logits.dtype).min)
    window = logits.shape[-1]
    selected = None
    if compressed_kv is not None and compressed_indices is not None:
        valid = compressed_indices >= 0
        selected = compressed_kv[rows, compressed_indices.clamp_min(0).long()]
        picked = torch.einsum("bhsd,bskd->bhsk", query, selected.to(query.dtype)) * scale
        picked = picked.masked_fill(~valid.unsqueeze(1), float("-inf"))
        logits = torch.cat((logits, picked), dim=-1)
    sink = sinks.float().view(1, -1, 1, 1).expand(batch, -1, length, -1)
    combined = torch.cat((logits.float(), sink), dim=-1)
    combined = combined - combined.max(dim=-1, keepdim=True).values
    probs = torch.softmax(combined, dim=-1)[..., :-1]
    probs = F.dropout(probs, dropout, dropout > 0).to(kv.dtype)
    out = torch.einsum("bhlw,blwd->bhld", probs[..., :window], window_kv)
    if selected is not None:
        out = out + torch.einsum("bhsk,bskd->bhsd", probs[..., window:], selected.to(probs.dtype))
    return out.transpose(1, 2).contiguous()


def _index_kernel_ok(query, keys, weights, width, candidates) -> bool:
    heads, dim = query.shape[2], query.shape[3]
    return (query.dtype == torch.bfloat16 and keys.dtype == torch.bfloat16 and dim in (64, 128)
            and 4 <= heads <= 64 and heads & (heads - 1) == 0 and width > 0
            and (candidates is None or candidates.numel() == query.shape[0] * query.shape[1] * width))


def index_scores(query, keys, weights, starts, ends, width, candidates=None):
    if on_gpu(query) and _index_kernel_ok(query, keys, weights, width, candidates):
        cand = None if candidates is None else candidates.bool().contiguous()
        return ext().index_scores(query.contiguous(), keys.contiguous(), weights.float().contiguous(),
                                  starts.to(torch.int32).contiguous(), ends.to(torch.int32).contiguous(),
                                  int(width), cand)
    return index_scores_reference(query, keys, weights, starts, ends, width, candidates)


def index_scores_reference(query, keys, weights, starts, ends, width, candidates=None):
    if width == 0:
        return query.new_empty((*query.shape[:2], 0), dtype=torch.float32)
    idx = starts.unsqueeze(-1) + torch.arange(width, device=query.device)
    valid = idx < ends.unsqueeze(-1)
    if candidates is not None:
        valid = valid & candidates
    rows = torch.arange(query.shape[0], device=query.device)[:, None, None]
    gathered = keys[rows, idx.clamp_max(keys.shape[1] - 1)]
    dots = torch.einsum("blhd,blkd->blkh", query.float(), gathered.float())
    scores = (dots.relu() * query.shape[-1] ** -0.5 * weights.float().unsqueeze(2)).sum(-1)
    return scores.masked_fill(~valid, float("-inf"))


__all__ = ["index_scores", "index_scores_reference", "sparse_attention", "sparse_attention_reference"]
