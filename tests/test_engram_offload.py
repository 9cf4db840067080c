"""Engram host-resident tables and the direct-mapped row cache (CPU, plus one GPU case).

Every lookup must return exactly ``weight[ids]`` whatever the slot collisions, the staging chunk
size or the history of the cache, and the backward must keep every occurrence.
"""

import pytest
import torch

from tiny_dsv41_b200.parallel.engram_offload import CPUEmbeddingLookup, RowCache, install_engram_sgd_hooks


def _table(rows=64, width=8, dtype=torch.float32, seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(rows, width, generator=g).to(dtype)


def _cache(weight, slots, device="cpu"):
    return RowCache(slots * (weight.shape[1] * weight.element_size() + 8), torch.device(device))


def test_colliding_ids_return_their_own_rows():
    weight = _table()
    cache = _cache(weight, 4)
    ids = torch.tensor([1, 5, 2, 9])  # 1, 5 and 9 share slot 1
    torch.testing.assert_close(cache.read(weight, ids), weight[ids], rtol=0, atol=0)
    # the slot keeps the last distinct id, so 9 hits and 1 / 5 miss on the next lookup
    cache.metrics.update(hits=0, misses=0)
    torch.testing.assert_close(cache.read(weight, torch.tensor([9, 1, 5, 2])), weight[[9, 1, 5, 2]], rtol=0, atol=0)
    assert cache.metrics["hits"] == 2 and cache.metrics["misses"] == 2


def test_random_lookups_with_small_staging_chunks(monkeypatch):
    weight = _table(rows=200, width=6)
    monkeypatch.setattr(RowCache, "STAGING_BYTES", 3 * 6 * 4)  # three rows per transfer
    cache = _cache(weight, 7)
    g = torch.Generator().manual_seed(1)
    for _ in range(30):
        ids = torch.randint(0, 200, (int(torch.randint(1, 40, (1,), generator=g)),), generator=g)
        torch.testing.assert_close(cache.read(weight, ids), weight[ids], rtol=0, atol=0)
    assert cache.metrics["hits"] + cache.metrics["misses"] > 0
    assert cache._ticket is None


def test_in_place_update_invalidates_and_new_table_rebinds():
    weight = _table()
    cache = _cache(weight, 8)
    ids = torch.tensor([3, 4, 3])
    cache.read(weight, ids)
    with torch.no_grad():
        weight.add_(1.0)  # bumps _version
    torch.testing.assert_close(cache.read(weight, ids), weight[ids], rtol=0, atol=0)
    other = _table(seed=3)
    torch.testing.assert_close(cache.read(other, ids), other[ids], rtol=0, atol=0)


def test_budget_below_one_row_is_rejected():
    weight = _table()
    with pytest.raises(ValueError):
        RowCache(8, torch.device("cpu")).read(weight, torch.tensor([0]))


def test_out_of_range_ids_are_rejected_and_cache_recovers():
    weight = _table()
    cache = _cache(weight, 4)
    with pytest.raises(IndexError):
        cache.read(weight, torch.tensor([1, 64]))
    torch.testing.assert_close(cache.read(weight, torch.tensor([1, 5])), weight[[1, 5]], rtol=0, atol=0)


def test_lookup_backward_keeps_occurrences_and_sgd_coalesces_in_fp32():
    weight = torch.nn.Parameter(_table(dtype=torch.bfloat16))
    lookup = CPUEmbeddingLookup()
    lookup.configure_cache(4 * (8 * 2 + 8), "cpu")
    ids = torch.tensor([[1, 5, 1], [9, 2, 5]])
    # two micro-batches: the accumulation hook concatenates them instead of adding in bf16
    for _ in range(2):
        rows = lookup(weight, ids, device="cpu")
        torch.testing.assert_close(rows, weight.detach()[ids], rtol=0, atol=0)
        rows.float().sum().backward()
    grad = weight.grad
    assert grad.is_sparse and grad._indices().shape[1] == 2 * ids.numel()

    class Table(torch.nn.Module):
        engram_offload = True
        sparse_gradients = True

        def __init__(self):
            super().__init__()
            self.weight = weight

        def synchronize(self):
            lookup.synchronize()

        def clear_cache(self):
            lookup.clear_cache()

    model = Table()
    opt = torch.optim.SGD([weight], lr=0.5)
    install_engram_sgd_hooks(model, opt)
    before = weight.detach().float().clone()
    opt.step()
    counts = torch.bincount(ids.reshape(-1), minlength=weight.shape[0]).float() * 2
    expected = before - 0.5 * counts[:, None]
    torch.testing.assert_close(weight.detach().float(), expected.to(torch.bfloat16).float(), rtol=0, atol=1e-2)
    # the step bumped the version and the hook invalidated the cache: fresh rows are served
    torch.testing.assert_close(lookup(weight, ids, device="cpu"), weight.detach()[ids], rtol=0, atol=0)


def test_second_lookup_in_one_backward_is_refused():
    weight = torch.nn.Parameter(_table(dtype=torch.bfloat16))
    lookup = CPUEmbeddingLookup()
    a = lookup(weight, torch.tensor([1, 2]), device="cpu")
    b = lookup(weight, torch.tensor([3]), device="cpu")
    with pytest.raises(RuntimeError, match="one lookup"):
        (a.float().sum() + b.float().sum()).backward()


@pytest.mark.gpu
def test_gpu_cache_colliding_ids_forward_backward():
    from tiny_dsv41_b200.parallel.engram_offload import CPUEmbeddingLookup as Lookup

    weight = torch.nn.Parameter(_table(rows=4096, width=256, dtype=torch.bfloat16))
    lookup = Lookup()
    lookup.configure_cache(64 * (256 * 2 + 8), "cuda")
    g = torch.Generator().manual_seed(2)
    for _ in range(6):
        ids = torch.randint(0, 4096, (3, 97), generator=g)
        ids[0, :4] = torch.tensor([1, 65, 129, 1])  # collide in slot 1 of 64
        rows = lookup(weight, ids.cuda(), device="cuda")
        torch.testing.assert_close(rows.cpu(), weight.detach()[ids], rtol=0, atol=0)
        rows.float().pow(2).sum().backward()
        grad = weight.grad.coalesce()
        dense = torch.zeros(4096, 256)
        dense.index_add_(0, ids.reshape(-1), 2 * weight.detach()[ids].reshape(-1, 256).float())
        torch.testing.assert_close(grad.to_dense().float(), dense, rtol=2e-2, atol=2e-2)
        weight.grad = None
    lookup.synchronize()
    metrics = lookup.cache_metrics
    assert metrics["hits"] > 0 and metrics["misses"] > 0
