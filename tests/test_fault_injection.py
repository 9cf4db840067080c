"""Host-side fault injection: non-finite gradients abort before the optimizer step, a rank whose
experts receive no tokens keeps the expert-parallel collectives in step, a failing rollout child
surfaces its traceback, and corrupted checkpoints are refused. No GPU is faulted."""

import json
import shutil
from pathlib import Path

import pytest
import torch

from tests.dist_utils import run_gloo

ROOT = Path(__file__).resolve().parents[1]


def test_sft_non_finite_gradient_aborts(tmp_path):
    from tiny_dsv41_b200.models.qwen import Qwen3MoeConfig, Qwen3MoeForCausalLM
    from tiny_dsv41_b200.runtime import Runtime
    from tiny_dsv41_b200.train.sft import train_update

    torch.manual_seed(0)
    model = Qwen3MoeForCausalLM(Qwen3MoeConfig.tiny(num_hidden_layers=2, max_window_layers=2, vocab_size=32))
    opt = torch.optim.SGD(model.parameters(), lr=1.0)
    before = {n: p.detach().clone() for n, p in model.named_parameters()}
    model.lm_head.weight.register_hook(lambda g: g * float("nan"))
    ids = torch.randint(0, 32, (1, 16))
    labels = ids.clone()
    batch = {"input_ids": ids, "labels": labels, "attention_mask": torch.ones_like(ids)}
    with pytest.raises(RuntimeError, match="non-finite"):
        train_update(model, opt, [batch], family="qwen", runtime=Runtime(torch.device("cpu")))
    for n, p in model.named_parameters():
        assert torch.equal(p, before[n]), n  # no parameter moved


def _empty_owner(rank, world):
    from torch.distributed.device_mesh import init_device_mesh

    from tiny_dsv41_b200.ops import gemm as G
    from tiny_dsv41_b200.ops import moe as M
    from tiny_dsv41_b200.parallel.dispatch import AllToAllTokenDispatcher

    mesh = init_device_mesh("cpu", (world,), mesh_dim_names=("ep",))
    disp = AllToAllTokenDispatcher(mesh)
    disp.expert_range(8)
    torch.manual_seed(rank)
    x = torch.randn(6, 16, requires_grad=True)
    ids = torch.randint(0, 4, (6, 2), dtype=torch.int32)  # every route lands on rank 0's experts
    w = torch.rand(6, 2, requires_grad=True)
    w1 = torch.randn(4, 8, 16, requires_grad=True)  # gate_up of this rank's 4 experts
    w2 = torch.randn(4, 16, 4, requires_grad=True)  # down
    batch = disp.dispatch(x, ids, w)
    h = M.swiglu(G.grouped_linear(batch.rows, w1, batch.offsets, batch.sizes), total=batch.total)
    out = disp.combine(G.grouped_linear(h, w2, batch.offsets, batch.sizes), batch)
    out.sum().backward()  # would deadlock if the empty owner skipped a backward exchange
    assert x.grad is not None and torch.isfinite(x.grad).all()


def test_expert_parallel_with_an_empty_owner():
    run_gloo(_empty_owner, 2)


def test_rollout_child_failure_surfaces(tmp_path):
    from tiny_dsv41_b200.rl.config import RLConfig
    from tiny_dsv41_b200.rl.runtime import run_training

    data = tmp_path / "d.jsonl"
    data.write_text(json.dumps({"prompt_ids": [1, 2, 3], "target_ids": [4]}) + "\n")
    cfg = RLConfig.from_dict(dict(max_steps=1, group_size=2, max_new_tokens=2, rollout_engine="native-pytorch",
                                  output_dir=str(tmp_path / "out"), reward="operator:truediv",
                                  worker_timeout_seconds=120))
    with pytest.raises(Exception) as info:
        run_training(model_dir=ROOT / "examples" / "tiny-dsv41", data_path=data, config=cfg, random_init=True)
    assert "rollout worker failed" in str(info.value) or "reward" in str(info.value).lower()


def test_corrupted_checkpoints_are_refused(tmp_path):
    from tiny_dsv41_b200.rl import checkpoint as ck

    class P(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.a = torch.nn.Linear(2, 2)

        def trainable_state_dict(self):
            return dict(self.a.state_dict())

        def frozen_state_dict(self):
            return {}

        def load_trainable_state_dict(self, s):
            self.a.load_state_dict(s)

        def load_frozen_state_dict(self, s):
            pass

    art = ck.publish_policy_artifact(P(), 1, tmp_path, lineage="x", identity={}, sampling={})
    raw = bytearray(Path(art["path"]).read_bytes())
    raw[-5] ^= 0xFF
    Path(art["path"]).chmod(0o644)
    Path(art["path"]).write_bytes(bytes(raw))
    with pytest.raises(ValueError):
        ck.load_policy_artifact(P(), art)


def test_status_monitor_is_inert_without_a_gpu():
    from tiny_dsv41_b200.ops import StatusMonitor

    monitor = StatusMonitor("cpu")
    assert not monitor.enabled
    monitor.step_end("cpu step")  # nothing to read, nothing raised


@pytest.mark.gpu
def test_peer_wait_timeout_surfaces_as_a_python_error():
    """A wait on a flag that no rank raises (one GPU, local memory) gives up after the runtime
    limit, records status 5, and the per-step monitor raises; the context stays usable."""
    import time

    from tiny_dsv41_b200 import ops

    ops.check_status("before the timeout test")
    previous = ops.peer_wait_limit()
    ops.set_peer_wait_limit(0.01)
    try:
        flags = torch.zeros(4, dtype=torch.int32, device="cuda")
        monitor = ops.StatusMonitor("cuda")
        start = time.perf_counter()
        ops.ext().ep_wait(flags, 1)
        with pytest.raises(ops.DeviceStatusError) as error:
            monitor.step_end("timeout test")
        assert error.value.code == 5
        assert time.perf_counter() - start < 2.0
        monitor.step_end("after the timeout")  # the word was reset
        flags.fill_(1)
        ops.ext().ep_wait(flags, 1)  # raised flags pass at once
        monitor.step_end("raised flags")
        assert torch.ones(8, device="cuda").sum().item() == 8
    finally:
        ops.set_peer_wait_limit(previous)
