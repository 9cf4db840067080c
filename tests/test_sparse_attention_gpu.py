"""DeepSeek-V4 sparse attention forward kernel (csrc/sparse_attention.cu) against the fp32
PyTorch restatement of the same op: sliding-window keys with a mask, selected compressed keys with
-1 holes, per-head sink logits, head groups of 64 with a partial last group."""

import pytest
import torch

from tiny_dsv41_b200 import ops
from tiny_dsv41_b200.ops.sparse_attention import sparse_attention, sparse_attention_reference

pytestmark = pytest.mark.gpu


def _case(batch, length, heads, dim, window, comp_rows, selected, seed=0, device="cuda"):
    gen = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn(batch, length, heads, dim, generator=gen).to(device, torch.bfloat16)
    kv = torch.randn(batch, length, dim, generator=gen).to(device, torch.bfloat16)
    pos = torch.arange(length).view(1, -1, 1)
    idx = pos - window + 1 + torch.arange(window).view(1, 1, -1)
    mask = (idx >= 0).expand(batch, -1, -1).clone()
    mask[:, ::7, 0] = False  # some extra holes
    win_idx = idx.clamp_min(0).expand(batch, -1, -1).contiguous()
    comp = sel = None
    if selected:
        comp = torch.randn(batch, comp_rows, dim, generator=gen).to(device, torch.bfloat16)
        sel = torch.randint(-1, comp_rows, (batch, length, selected), generator=gen)
    sinks = torch.randn(heads, generator=gen)
    to = lambda t: None if t is None else t.to(device)
    return (q.transpose(1, 2), kv, to(win_idx), to(mask), comp, to(sel), sinks.to(device))


@pytest.mark.parametrize("dim", [128, 256, 512])
@pytest.mark.parametrize("heads", [64, 80])
def test_sparse_attention_forward_matches_fp32(dim, heads):
    q, kv, widx, wmask, comp, sel, sinks = _case(2, 67, heads, dim, 32, 45, 40)
    out = sparse_attention(q, kv, widx, wmask, comp, sel, sinks)
    torch.cuda.synchronize()
    ops.check_status("sparse_attention")
    ref = sparse_attention_reference(q.float(), kv.float(), widx, wmask, comp.float(), sel, sinks)
    assert out.shape == ref.shape
    torch.testing.assert_close(out.float(), ref, atol=2e-2, rtol=2e-2)


def test_sparse_attention_window_only_and_lse():
    q, kv, widx, wmask, _, _, sinks = _case(1, 150, 64, 512, 128, 0, 0, seed=3)
    out, lse = ops.ext().sparse_attention_fwd(q.transpose(1, 2).contiguous(), kv, widx, wmask, None, None, sinks)
    ref = sparse_attention_reference(q.float(), kv.float(), widx, wmask, None, None, sinks)
    torch.testing.assert_close(out.float(), ref, atol=2e-2, rtol=2e-2)
    # lse over window logits and the sink, natural log
    rows = torch.arange(1, device=q.device).view(-1, 1, 1)
    wk = kv.float()[rows, widx]
    logits = torch.einsum("bhld,blwd->blhw", q.float(), wk) * 512 ** -0.5
    logits = logits.masked_fill(~wmask.unsqueeze(2), float("-inf"))
    full = torch.cat((logits, sinks.view(1, 1, -1, 1).expand(1, 150, -1, 1)), dim=-1)
    torch.testing.assert_close(lse, torch.logsumexp(full, dim=-1), atol=1e-2, rtol=1e-3)


@pytest.mark.parametrize("dim", [128, 256, 512])
@pytest.mark.parametrize("heads", [64, 80])
def test_sparse_attention_backward_matches_fp32(dim, heads):
    q, kv, widx, wmask, comp, sel, sinks = _case(2, 53, heads, dim, 32, 37, 40, seed=11)
    gen = torch.Generator(device="cpu").manual_seed(12)
    dout = torch.randn(2, 53, heads, dim, generator=gen).to("cuda", torch.bfloat16)
    leaves = [t.detach().requires_grad_() for t in (q, kv, comp, sinks)]
    out = sparse_attention(leaves[0], leaves[1], widx, wmask, leaves[2], sel, leaves[3])
    out.backward(dout)
    torch.cuda.synchronize()
    ops.check_status("sparse_attention backward")
    ref_leaves = [t.detach().float().requires_grad_() for t in (q, kv, comp, sinks)]
    ref = sparse_attention_reference(ref_leaves[0], ref_leaves[1], widx, wmask, ref_leaves[2], sel, ref_leaves[3])
    ref.backward(dout.float())
    for name, got, want in zip(("dq", "dkv", "dcompressed", "dsinks"), leaves, ref_leaves):
        g, w = got.grad.float(), want.grad
        err = (g - w).norm() / w.norm().clamp_min(1e-6)
        assert err < 2e-2, f"{name}: relative error {err:.3e}"


@pytest.mark.parametrize("dim", [128, 512])
def test_sparse_attention_deterministic_backward(dim, monkeypatch):
    """Ordered KV gradients: equal to the fp32 restatement and bitwise equal across runs, also with
    token chunks smaller than the sequence."""
    from tiny_dsv41_b200.ops import sparse_attention as sa

    monkeypatch.setattr(sa, "_EDGE_BUFFER_BYTES", 16 * (48 + 12) * 2 * dim * 4)  # ~16-token chunks
    q, kv, widx, wmask, comp, sel, sinks = _case(2, 45, 80, dim, 48, 29, 12, seed=21)
    gen = torch.Generator(device="cpu").manual_seed(22)
    dout = torch.randn(2, 45, 80, dim, generator=gen).to("cuda", torch.bfloat16)
    runs = []
    for _ in range(3):
        leaves = [t.detach().requires_grad_() for t in (q, kv, comp, sinks)]
        out = sparse_attention(leaves[0], leaves[1], widx, wmask, leaves[2], sel, leaves[3], deterministic=True)
        out.backward(dout)
        runs.append([t.grad.clone() for t in leaves])
    torch.cuda.synchronize()
    ops.check_status("sparse_attention deterministic backward")
    for other in runs[1:]:
        for a, b in zip(runs[0], other):
            assert torch.equal(a, b)
    ref_leaves = [t.detach().float().requires_grad_() for t in (q, kv, comp, sinks)]
    ref = sparse_attention_reference(ref_leaves[0], ref_leaves[1], widx, wmask, ref_leaves[2], sel, ref_leaves[3])
    ref.backward(dout.float())
    for name, got, want in zip(("dq", "dkv", "dcompressed", "dsinks"), runs[0], ref_leaves):
        err = (got.float() - want.grad).norm() / want.grad.norm().clamp_min(1e-6)
        assert err < 2e-2, f"{name}: relative error {err:.3e}"
