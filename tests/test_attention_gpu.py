"""tcgen05 flash attention (csrc/attention.cu) against a plain fp32 PyTorch restatement."""

import math

import pytest
import torch

from tiny_dsv41_b200 import ops
from tiny_dsv41_b200.ops import attention as A

pytestmark = pytest.mark.gpu


def reference(q, k, v):
    """fp32 causal GQA attention on [B, L, H, D] inputs; returns (out, lse [B, H, L])."""
    qf, kf, vf = (t.float().transpose(1, 2) for t in (q, k, v))
    groups = qf.shape[1] // kf.shape[1]
    kf = kf.repeat_interleave(groups, dim=1)
    vf = vf.repeat_interleave(groups, dim=1)
    s = qf @ kf.transpose(-1, -2) / math.sqrt(q.shape[-1])
    length = q.shape[1]
    mask = torch.ones(length, length, dtype=torch.bool, device=q.device).tril()
    s = s.masked_fill(~mask, float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    out = torch.softmax(s, dim=-1) @ vf
    return out.transpose(1, 2), lse


def _inputs(batch, seq, heads, kv_heads, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(batch, seq, heads, 128, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(batch, seq, kv_heads, 128, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(batch, seq, kv_heads, 128, device="cuda", generator=g).to(torch.bfloat16)
    return q, k, v


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


# the default one-head kernel, and the opt-in two-heads-per-CTA kernel (even GQA groups only)
@pytest.mark.parametrize("two_heads", [False, True])
@pytest.mark.parametrize("batch,seq,heads,kv_heads",
                         [(1, 128, 2, 1), (1, 512, 4, 2), (2, 384, 8, 1), (1, 256, 3, 1), (2, 640, 32, 4)])
def test_attention_forward(batch, seq, heads, kv_heads, two_heads, monkeypatch):
    monkeypatch.setenv("TDSV_ATTN_FWD2", "1" if two_heads else "0")
    q, k, v = _inputs(batch, seq, heads, kv_heads)
    out, lse = ops.ext().attn_fwd(q, k, v)
    ops.check_status("attn_fwd")
    ref_out, ref_lse = reference(q, k, v)
    assert torch.allclose(lse, ref_lse, atol=2e-3, rtol=1e-3), (lse - ref_lse).abs().max().item()
    assert _rel(out, ref_out) < 1e-2
    assert (out.float() - ref_out).abs().max().item() < 5e-2


@pytest.mark.parametrize("batch,seq,heads,kv_heads", [(1, 128, 2, 1), (1, 512, 4, 2), (2, 384, 8, 1)])
def test_attention_backward(batch, seq, heads, kv_heads):
    q, k, v = _inputs(batch, seq, heads, kv_heads, seed=1)
    dout = torch.randn(batch, seq, heads, 128, device="cuda").to(torch.bfloat16)
    qr, kr, vr = (t.float().requires_grad_() for t in (q, k, v))
    ref_out, _ = reference(qr, kr, vr)
    ref_dq, ref_dk, ref_dv = torch.autograd.grad(ref_out, (qr, kr, vr), dout.float())
    qa, ka, va = (t.clone().requires_grad_() for t in (q, k, v))
    out = A.causal_attention(qa, ka, va)
    out.backward(dout)
    ops.check_status("attn_bwd")
    assert _rel(out, ref_out) < 1e-2
    for got, want in ((qa.grad, ref_dq), (ka.grad, ref_dk), (va.grad, ref_dv)):
        assert got.dtype == torch.bfloat16 and got.shape == want.shape
        assert _rel(got, want) < 2e-2


def test_attention_matches_sdpa_at_model_shape():
    """Qwen3-30B-A3B attention shape (32 q / 4 kv heads) at a 1k sequence against cuDNN SDPA."""
    q, k, v = _inputs(1, 1024, 32, 4, seed=2)
    out = A.flash_attention(q, k, v)
    ref = A.sdpa_attention(q, k, v)
    ops.check_status("attn_fwd")
    assert _rel(out, ref) < 1e-2


def test_attention_backward_matches_sdpa_at_4k():
    """Full benchmark shape (L 4096, 32 q / 4 kv heads): forward and gradients against cuDNN SDPA."""
    q, k, v = _inputs(1, 4096, 32, 4, seed=3)
    dout = torch.randn_like(q)
    grads = []
    for fn in (A.flash_attention, A.sdpa_attention):
        leaves = [t.clone().requires_grad_() for t in (q, k, v)]
        out = fn(*leaves)
        out.backward(dout)
        grads.append([out] + [t.grad for t in leaves])
    ops.check_status("attention 4k")
    for got, want in zip(*grads):
        assert _rel(got, want) < 2e-2
