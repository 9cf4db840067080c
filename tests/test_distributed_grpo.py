"""Distributed query-LoRA GRPO on CPU: two gloo learner ranks against the native rollout service
over the authenticated LoRA RPC (the same protocol as the external vLLM service)."""

import json
import os
import secrets
import shutil
import socket
import threading
from pathlib import Path

import pytest
import torch

from tests.dist_utils import run_gloo

ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.fixture()
def service(tmp_path):
    from tiny_dsv41_b200.models.dsv4 import DeepSeekV41Config, DeepSeekV41ForCausalLM
    from tiny_dsv41_b200.models.dsv4.checkpoint import write_released_checkpoint
    from tiny_dsv41_b200.rl.lora_config import DistributedLoRAConfig
    from tiny_dsv41_b200.rollout.native_service import NativeRolloutController
    from tiny_dsv41_b200.rollout.remote import RemoteLoRAServer

    torch.manual_seed(0)
    model_dir = tmp_path / "model"
    write_released_checkpoint(DeepSeekV41ForCausalLM(DeepSeekV41Config.tiny()), model_dir)
    for name in ("tokenizer.json", "tokenizer_config.json"):
        shutil.copy(ROOT / "examples" / "tiny-dsv41" / name, model_dir / name)
    token = secrets.token_hex(20)
    port = _free_port()
    controller = NativeRolloutController(model_dir, DistributedLoRAConfig(8, 16.0, (0, 2)))
    server = RemoteLoRAServer(("127.0.0.1", port), token, controller)
    thread = threading.Thread(target=server.serve_forever, daemon=True)
    thread.start()
    yield model_dir, port, token, controller
    server.shutdown()
    server.server_close()


def _learner(rank, world, args_list, token):
    os.environ["DSV41_ROLLOUT_TOKEN"] = token
    from tiny_dsv41_b200.rl.distributed_grpo import parse_args, run

    run(parse_args(args_list))


def test_distributed_grpo_two_ranks(service, tmp_path):
    model_dir, port, token, controller = service
    data = tmp_path / "train.jsonl"
    test = tmp_path / "test.jsonl"
    for path, rows in ((data, 6), (test, 2)):
        with path.open("w") as f:
            for i in range(rows):
                f.write(json.dumps({"prompt_ids": [1, 3, 8 + (i + (0 if path == data else 5)) % 9, 6, 4],
                                    "target_ids": [9, 10, 11]}) + "\n")
    out = tmp_path / "run"
    args = ["--model-dir", str(model_dir), "--train-jsonl", str(data), "--test-jsonl", str(test), "--output-dir",
            str(out), "--rollout-port", str(port), "--reward", "token_accuracy", "--group-size", "4",
            "--learner-microbatch-size", "2", "--updates", "2", "--max-new-tokens", "3", "--temperature", "1.0",
            "--lora-rank", "8", "--lora-alpha", "16", "--lora-layers", "0,2", "--learning-rate", "1e-2",
            "--device", "cpu", "--rollout-correction", "decoupled-token-tis"]
    run_gloo(_learner, 2, args, token)
    summary = json.loads((out / "summary.json").read_text())
    assert summary["status"] == "completed" and summary["optimizer_updates"] == 2
    updates = [json.loads(line) for line in (out / "updates.jsonl").read_text().splitlines()]
    assert [u["policy_ack"]["version"] for u in updates] == [1, 2]
    assert all(u["changed_adapter_elements"] > 0 for u in updates)
    assert [r["version"] for r in controller.activation_receipts] == [0, 1, 2]
