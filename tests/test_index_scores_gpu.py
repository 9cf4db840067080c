"""tcgen05 sparse-indexer scores (csrc/index_scores.cu) against the PyTorch restatement."""

import pytest
import torch

from tiny_dsv41_b200 import ops
from tiny_dsv41_b200.ops import sparse_attention as S

pytestmark = pytest.mark.gpu


def _case(batch, seq, heads, dim, key_len, packed, with_candidates, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    query = torch.randn(batch, seq, heads, dim, device="cuda", generator=g).to(torch.bfloat16)
    keys = torch.randn(batch, key_len, dim, device="cuda", generator=g).to(torch.bfloat16)
    weights = torch.randn(batch, seq, heads, device="cuda", generator=g) * heads ** -0.5
    pos = torch.arange(seq, device="cuda")
    if packed:  # two packed sequences per row: the second one's keys start half way
        half = seq // 2
        starts = torch.where(pos < half, 0, key_len // 2).expand(batch, seq).contiguous()
        visible = torch.where(pos < half, pos, pos - half) // 2 + 1
    else:
        starts = torch.zeros(batch, seq, dtype=torch.long, device="cuda")
        visible = pos // 2 + 1
    ends = torch.minimum(starts + visible, torch.full_like(starts, key_len))
    width = int((ends - starts).max().item()) + 3
    candidates = None
    if with_candidates:
        candidates = torch.rand(batch, seq, width, device="cuda", generator=g) > 0.3
    return query, keys, weights, starts, ends, width, candidates


@pytest.mark.parametrize("batch,seq,heads,dim,key_len,packed,cand", [
    (1, 37, 4, 64, 20, False, False),    # tiny-config shape (4 index heads x 64), partial query block
    (2, 96, 4, 64, 48, True, True),
    (1, 300, 32, 128, 160, True, False),  # DeepSeek-V4-Flash indexer heads (32 x 128)
    (2, 256, 32, 128, 300, False, True),
])
def test_index_scores_match_reference(batch, seq, heads, dim, key_len, packed, cand):
    args = _case(batch, seq, heads, dim, key_len, packed, cand)
    got = S.index_scores(*args)
    ops.check_status("index_scores")
    want = S.index_scores_reference(*args)
    assert got.shape == want.shape
    finite = torch.isfinite(want)
    assert torch.equal(finite, torch.isfinite(got))
    scale = want[finite].abs().max().clamp_min(1e-6)
    assert ((got[finite] - want[finite]).abs().max() / scale).item() < 1e-3
