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


def test_sparse_attention_backward_runs_through_restatement():
    q, kv, widx, wmask, comp, sel, sinks = _case(1, 40, 64, 128, 16, 20, 12, seed=5)
    leaves = [t.detach().requires_grad_() for t in (q, kv, comp, sinks)]
    out = sparse_attention(leaves[0], leaves[1], widx, wmask, leaves[2], sel, leaves[3])
    out.float().square().sum().backward()
    for t in leaves:
        assert t.grad is not None and torch.isfinite(t.grad).all()
