"""A training step replayed as one captured CUDA graph (QwenTrainer(cuda_graph=True)) against the
same steps run eagerly: same losses step by step, same parameters at the end. Covers the device-side
step counters of both optimizers and the peer-memory dense sync (world 1) inside the graph."""

import pytest
import torch

from tiny_dsv41_b200 import ops
from tiny_dsv41_b200.models.qwen import Qwen3MoeConfig

pytestmark = pytest.mark.gpu


def _run(cuda_graph: bool, batches):
    from tiny_dsv41_b200.train.qwen_sft import QwenTrainer

    cfg = Qwen3MoeConfig.tiny(num_hidden_layers=2, vocab_size=512)
    trainer = QwenTrainer(cfg, lr=3e-3, seed=3, tokens_per_rank=256, cuda_graph=cuda_graph, graph_warmup=2)
    losses = [float(trainer.train_step(ids, labels).item()) for ids, labels in batches]
    torch.cuda.synchronize()
    ops.check_status("cuda graph step")
    params = {n: p.detach().float().clone() for n, p in trainer.model.named_parameters()}
    captured = trainer._graph is not None
    trainer.close()
    return losses, params, captured


def test_cuda_graph_step_matches_eager():
    gen = torch.Generator().manual_seed(0)
    ids = torch.randint(0, 512, (1, 256), generator=gen)
    labels = ids.clone()
    labels[:, :128] = -100
    batches = [(ids.pin_memory(), labels.pin_memory())] * 6  # one batch: the loss must fall
    eager, p_eager, cap0 = _run(False, batches)
    graph, p_graph, cap1 = _run(True, batches)
    assert not cap0 and cap1
    assert eager[-1] < eager[0], eager
    for a, b in zip(eager, graph):
        assert abs(a - b) <= 2e-3 * abs(a), (eager, graph)
    for name, p in p_eager.items():
        q = p_graph[name]
        err = ((p - q).norm() / p.norm().clamp_min(1e-12)).item()
        assert err < 2e-2, (name, err)
