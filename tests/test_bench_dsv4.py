"""The DeepSeek-V4.1-Flash LoRA SFT harness (bench_dsv4.py) at the tiny
configuration on CPU: the synthetic backbone (frozen MXFP4 experts, Engram offload, mHC), LoRA on
the query projections, one and two gloo ranks (EP2)."""

import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ARGS = ["--config", "tiny", "--seq-len", "64", "--steps", "1", "--warmup", "1", "--device", "cpu"]


def _record(out: str) -> dict:
    lines = [line for line in out.splitlines() if line.startswith("{")]
    assert lines, out[-2000:]
    return json.loads(lines[-1])


def test_flash_expert_memory_needs_eight_gpus():
    sys.path.insert(0, ROOT)
    import bench_dsv4
    from tiny_dsv41_b200.models.dsv4 import DeepSeekV41Config

    cfg = DeepSeekV41Config.from_json(bench_dsv4.CONFIGS["flash"])
    assert cfg.num_hidden_layers == 40 and cfg.n_routed_experts == 384 and cfg.hidden_size == 5120
    budget = bench_dsv4.HBM_BYTES - bench_dsv4.ACTIVATION_RESERVE
    assert bench_dsv4.expert_bytes_per_rank(cfg, 1) > budget
    assert 30 * 2 ** 30 < bench_dsv4.expert_bytes_per_rank(cfg, 8) < 40 * 2 ** 30


def test_single_rank_step():
    out = subprocess.run([sys.executable, "bench_dsv4.py", "--layers", "2", *ARGS], cwd=ROOT, capture_output=True,
                         text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-3000:]
    record = _record(out.stdout)
    assert record["value"] > 0 and record["config"]["parallelism"] == "ep1"
    assert record["adapter_parameters"] > 0 and record["loss"] == record["loss"]  # finite (not NaN)


@pytest.mark.timeout(600)
def test_two_rank_expert_parallel_step():
    env = dict(os.environ, OMP_NUM_THREADS="2")
    out = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                          "--master-addr", "127.0.0.1", "--master-port", "29733", "bench_dsv4.py", "--layers", "3",
                          *ARGS], cwd=ROOT, capture_output=True, text=True, timeout=600, env=env)
    assert out.returncode == 0, out.stderr[-3000:]
    record = _record(out.stdout)
    assert record["value"] > 0 and record["config"]["parallelism"] == "ep2" and record["config"]["global_batch"] == 2


def test_synthetic_backbone_layout():
    """The loader's layout without a checkpoint: fp32 islands, bf16 elsewhere, packed experts with
    E8M0 scale 2^-6, Engram tables in host memory under offload, no meta tensors left."""
    import torch

    from tiny_dsv41_b200.models.dsv4 import DeepSeekV41Config
    from tiny_dsv41_b200.models.dsv4.checkpoint import prefix_config
    from tiny_dsv41_b200.models.dsv4.synthetic import build_synthetic_backbone

    sys.path.insert(0, ROOT)
    import bench_dsv4

    cfg = prefix_config(DeepSeekV41Config.from_json(bench_dsv4.CONFIGS["tiny"]), 2)
    model = build_synthetic_backbone(cfg, device="cpu", dtype=torch.bfloat16, engram_offload=True,
                                     sparse_engram_gradients=True, fp4_experts=True, seed=3)
    for name, p in model.named_parameters():
        island = any(key in name for key in ("attention_hc.", "moe_hc.", "attention.sinks.", "selection_bias"))
        assert p.dtype == (torch.float32 if island else torch.bfloat16), name
    routed = model.model.layers[0].moe.routed
    assert routed.frozen_fp4 and routed.gate_up_fp4.dtype == torch.uint8
    assert bool((routed.gate_up_scale == 121).all()) and routed.gate_up_fp4.float().std() > 50
    assert all(t.weight.device.type == "cpu" for t in model.model.engram_tables.values())
    norms = [p for n, p in model.named_parameters() if n.endswith("input_norm.weight")]
    assert norms and all(bool((p == 1).all()) for p in norms)
