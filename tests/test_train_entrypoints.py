"""Root training entry points on CPU: train.py (DCP resume), train_qwen.py (EP2 x FSDP2 on gloo)
and train_dsv4_checkpoint.py (released-layout checkpoint, plain and in-backward SGD)."""

import json
import shutil
from pathlib import Path

import pytest
import torch

from tests.dist_utils import run_gloo

ROOT = Path(__file__).resolve().parents[1]


def test_tiny_train_resume_matches_uninterrupted(tmp_path, capsys):
    from tiny_dsv41_b200.train.tiny import main

    def losses(text):
        return {r["step"]: r["loss"] for r in map(json.loads, (l for l in text.splitlines() if l.startswith('{"step"')))}

    main(["--steps", "4", "--device", "cpu", "--output-dir", str(tmp_path / "a"), "--seq-len", "16"])
    straight = losses(capsys.readouterr().out)
    main(["--steps", "2", "--device", "cpu", "--output-dir", str(tmp_path / "b"), "--seq-len", "16"])
    main(["--steps", "4", "--device", "cpu", "--output-dir", str(tmp_path / "b"), "--seq-len", "16", "--resume"])
    resumed = losses(capsys.readouterr().out)
    assert resumed[3] == pytest.approx(straight[3], rel=1e-6)
    assert resumed[4] == pytest.approx(straight[4], rel=1e-6)
    assert (tmp_path / "b" / "checkpoint" / "step-4" / ".metadata").is_file()


@pytest.fixture(scope="module")
def qwen_dir(tmp_path_factory):
    from tiny_dsv41_b200.models.qwen import Qwen3MoeConfig, Qwen3MoeForCausalLM, save_qwen3_moe

    root = tmp_path_factory.mktemp("qwen") / "model"
    torch.manual_seed(0)
    save_qwen3_moe(Qwen3MoeForCausalLM(Qwen3MoeConfig.tiny(num_hidden_layers=2, max_window_layers=2)), root)
    return root


def _qwen(rank, world, model, out, ep):
    from tiny_dsv41_b200.runtime import initialize_runtime
    from tiny_dsv41_b200.train.qwen_cli import parse_args, train

    args = parse_args(["--model-path", str(model), "--steps", "2", "--seq-len", "32", "--device", "cpu",
                       "--ep-size", str(ep), "--metrics-file", str(out)])
    train(args, initialize_runtime("cpu", require_distributed=True))


def test_train_qwen_ep2(qwen_dir, tmp_path):
    run_gloo(_qwen, 2, qwen_dir, tmp_path / "m.json", 2)
    metrics = json.loads((tmp_path / "m.json").read_text())
    assert metrics["world_size"] == 2 and metrics["ep_size"] == 2 and metrics["parameter_delta_max"] > 0
    assert metrics["loss"] > 0 and metrics["grad_norm"] > 0


def _dsv4(rank, world, model, out, extra):
    from tiny_dsv41_b200.runtime import initialize_runtime
    from tiny_dsv41_b200.train.dsv4_cli import parse_args, train

    args = parse_args(["--model-path", str(model), "--steps", "2", "--num-layers", "2", "--seq-len", "16",
                       "--device", "cpu", "--ep-size", str(world), "--metrics-file", str(out), *extra])
    train(args, initialize_runtime("cpu", require_distributed=True))


@pytest.mark.parametrize("extra", [[], ["--optimizer-in-backward", "--sequence-packing", "--batch-size", "2"]])
def test_train_dsv4_checkpoint(tmp_path, extra):
    from tiny_dsv41_b200.models.dsv4 import DeepSeekV41Config, DeepSeekV41ForCausalLM
    from tiny_dsv41_b200.models.dsv4.checkpoint import write_released_checkpoint

    torch.manual_seed(0)
    write_released_checkpoint(DeepSeekV41ForCausalLM(DeepSeekV41Config.tiny()), tmp_path / "model")
    shutil.copy(ROOT / "examples" / "tiny-dsv41" / "tokenizer.json", tmp_path / "model" / "tokenizer.json")
    run_gloo(_dsv4, 1, tmp_path / "model", tmp_path / "m.json", extra)
    metrics = json.loads((tmp_path / "m.json").read_text())
    assert metrics["parameter_delta_max"] > 0 and metrics["loss"] > 0
    assert metrics["model"] == "DeepSeek-V4.1 2-layer prefix"
