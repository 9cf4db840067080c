"""SFT driver on CPU: full and LoRA runs, same-topology snapshot resume, and EP2 x FSDP2 on two
gloo ranks matching the single-process losses."""

import json
import shutil
from pathlib import Path

import pytest
import torch

from tests.dist_utils import run_gloo

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def qwen_dir(tmp_path_factory):
    from tiny_dsv41_b200.models.qwen import Qwen3MoeConfig, Qwen3MoeForCausalLM, save_qwen3_moe

    root = tmp_path_factory.mktemp("sft")
    torch.manual_seed(0)
    cfg = Qwen3MoeConfig.tiny(num_hidden_layers=2, max_window_layers=2, vocab_size=32)
    save_qwen3_moe(Qwen3MoeForCausalLM(cfg), root / "model")
    for name in ("tokenizer.json", "tokenizer_config.json"):
        shutil.copy(ROOT / "examples" / "tiny-dsv41" / name, root / "model" / name)
    with (root / "data.jsonl").open("w") as f:
        for a, b in [(1, 2), (2, 3), (3, 4), (4, 5)]:
            f.write(json.dumps({"prompt": f"what is the sum of {a} and {b}", "answer": f"{a + b} <eos>"}) + "\n")
    return root


def _args(root, out, *extra):
    from tiny_dsv41_b200.train.sft import parse_args

    return parse_args(["--model-path", str(root / "model"), "--data", str(root / "data.jsonl"), "--output-dir",
                       str(out), "--family", "qwen", "--batch-size", "1", "--seq-len", "64", "--learning-rate",
                       "1e-3", "--device", "cpu", *extra])


def _losses(out):
    rows = [json.loads(line) for line in (Path(out) / "metrics.jsonl").read_text().splitlines()]
    return [r["loss"] for r in rows if r["event"] == "train"], rows[-1]


def _single(rank, world, root, out, extra):
    from tiny_dsv41_b200.runtime import initialize_runtime
    from tiny_dsv41_b200.train.sft import train

    train(_args(root, out, *extra), initialize_runtime("cpu", require_distributed=True))


def test_full_sft_snapshot_resume(qwen_dir, tmp_path):
    out = tmp_path / "full"
    run_gloo(_single, 1, qwen_dir, out, ["--mode", "full", "--optimizer", "adamw", "--steps", "3"])
    losses, summary = _losses(out)
    assert len(losses) == 3 and losses[-1] < losses[0]
    manifest = json.loads((out / "checkpoint-00000003" / "manifest.json").read_text())
    assert manifest["step"] == 3 and manifest["world_size"] == 1
    run_gloo(_single, 1, qwen_dir, out, ["--mode", "full", "--optimizer", "adamw", "--steps", "4", "--resume",
                                         str(out / "checkpoint-00000003")])
    rows = [json.loads(line) for line in (out / "metrics.jsonl").read_text().splitlines()]
    loaded = [r for r in rows if r["event"] == "loaded"]
    assert loaded[1]["step"] == 3
    assert loaded[1]["eval_loss_before"] == pytest.approx(summary["eval_loss_after"], rel=1e-6)


def test_lora_sft_writes_adapter(qwen_dir, tmp_path):
    from tiny_dsv41_b200.lora import read_adapter

    out = tmp_path / "lora"
    run_gloo(_single, 1, qwen_dir, out, ["--mode", "lora", "--steps", "2", "--lora-rank", "4"])
    adapter = read_adapter(out / "adapter.pt")
    assert any(k.endswith("lora_a") for k in adapter["weights"])
    assert json.loads((out / "adapter_metadata.json").read_text())["step"] == 2


def test_ep2_fsdp2_matches_single_process(qwen_dir, tmp_path):
    extra = ["--mode", "full", "--optimizer", "adamw", "--steps", "3", "--no-save"]
    run_gloo(_single, 1, qwen_dir, tmp_path / "one", extra + ["--batch-size", "2"])
    run_gloo(_single, 2, qwen_dir, tmp_path / "two", extra + ["--ep-size", "2"])
    # one process sees both examples of a step as one batch of two; two ranks see one each
    a, _ = _losses(tmp_path / "one")
    b, _ = _losses(tmp_path / "two")
    assert b == pytest.approx(a, rel=1e-5)


@pytest.fixture(scope="module")
def dsv4_dir(tmp_path_factory):
    from tiny_dsv41_b200.models.dsv4 import DeepSeekV41Config, DeepSeekV41ForCausalLM
    from tiny_dsv41_b200.models.dsv4.checkpoint import write_released_checkpoint

    root = tmp_path_factory.mktemp("dsv4sft")
    torch.manual_seed(0)
    write_released_checkpoint(DeepSeekV41ForCausalLM(DeepSeekV41Config.tiny()), root / "model")
    for name in ("tokenizer.json", "tokenizer_config.json"):
        shutil.copy(ROOT / "examples" / "tiny-dsv41" / name, root / "model" / name)
    with (root / "data.jsonl").open("w") as f:
        for a, b in [(1, 2), (2, 3), (3, 4), (4, 5)]:
            f.write(json.dumps({"prompt": f"what is the sum of {a} and {b}", "answer": f"{a + b} <eos>"}) + "\n")
    return root


def _dsv4(rank, world, root, out, extra):
    from tiny_dsv41_b200.runtime import initialize_runtime
    from tiny_dsv41_b200.train.sft import parse_args, train

    args = parse_args(["--model-path", str(root / "model"), "--data", str(root / "data.jsonl"), "--output-dir",
                       str(out), "--family", "dsv4", "--batch-size", "1", "--seq-len", "64", "--learning-rate",
                       "5e-2", "--device", "cpu", "--mode", "full", "--optimizer", "sgd", "--engram-offload",
                       *extra])
    train(args, initialize_runtime("cpu", require_distributed=True))


def test_dsv4_full_sft_engram_rows_resume(dsv4_dir, tmp_path):
    run_gloo(_dsv4, 1, dsv4_dir, tmp_path / "a", ["--steps", "3"])
    run_gloo(_dsv4, 1, dsv4_dir, tmp_path / "b", ["--steps", "1"])
    snap = torch.load(tmp_path / "b" / "checkpoint-00000001" / "rank-00000.pt", weights_only=False)
    rows = snap["engram_rows"]["tables"]
    assert rows and all(r["indices"].numel() > 0 for r in rows.values())
    assert not any(".engram_tables." in n for n in snap["parameters"])
    run_gloo(_dsv4, 1, dsv4_dir, tmp_path / "b", ["--steps", "3", "--resume", str(tmp_path / "b" / "checkpoint-00000001")])
    a, sa = _losses(tmp_path / "a")
    b, sb = _losses(tmp_path / "b")
    assert b[-2:] == pytest.approx(a[-2:], rel=1e-5)
    steps = [json.loads(line) for line in (tmp_path / "a" / "metrics.jsonl").read_text().splitlines()]
    step = next(r for r in steps if r["event"] == "train")
    # offloaded Engram rows are looked up on the CPU path (no GPU row cache): the counters exist
    assert {"seconds", "engram_cache_hits", "engram_cache_misses", "engram_cache_transferred_rows"} <= set(step)
    assert sb["eval_loss_after"] == pytest.approx(sa["eval_loss_after"], rel=1e-5)


def test_dsv4_lora_engram_bundle(dsv4_dir, tmp_path):
    from tiny_dsv41_b200.rl.config import RLConfig
    from tiny_dsv41_b200.train.sft_export import resolve_initial_bundle

    out = tmp_path / "lora"
    run_gloo(_dsv4, 1, dsv4_dir, out, ["--steps", "2", "--mode", "lora", "--train-engram"])
    bundle = out / "sft-bundle-00000002"
    manifest = json.loads((bundle / "manifest.json").read_text())
    assert manifest["kind"] == "lora-engram-sft" and manifest["step"] == 2
    delta = torch.load(bundle / "engram_delta.pt", weights_only=True)
    assert all(t["indices"].numel() > 0 for t in delta["tables"].values())
    cfg = RLConfig.from_dict(dict(trainable_scope="lora", initial_adapter=str(bundle), rollout_engine="native-pytorch"))
    resolved = resolve_initial_bundle(cfg)
    assert resolved.initial_adapter.endswith("adapter.pt") and resolved.initial_engram_delta.endswith("engram_delta.pt")


def _dsv4_fsdp(rank, world, root, out, dump):
    import torch.distributed as dist

    from tiny_dsv41_b200.runtime import initialize_runtime
    from tiny_dsv41_b200.train import sft

    captured = {}
    original = sft.load_model

    def load_model(args, runtime):
        model, meshes = original(args, runtime)
        captured["model"] = model
        return model, meshes

    sft.load_model = load_model
    args = sft.parse_args(["--model-path", str(root / "model"), "--data", str(root / "data.jsonl"), "--output-dir",
                           str(out), "--family", "dsv4", "--batch-size", "1", "--seq-len", "64", "--learning-rate",
                           "1e-2", "--device", "cpu", "--mode", "full", "--optimizer", "adamw", "--steps", "1",
                           "--ep-size", "2"])
    sft.train(args, initialize_runtime("cpu", require_distributed=True))
    full = {}
    for name, value in captured["model"].state_dict().items():
        full[name] = value.full_tensor() if hasattr(value, "full_tensor") else value
    if rank == 0:
        torch.save({k: v for k, v in full.items() if ".routed." not in k and ".engram_tables." not in k}, dump)
    # experts (EP) and Engram rows (row-sharded) are rank-local slices of the global tensor
    torch.save({k: v for k, v in full.items() if ".routed." in k or ".engram_tables." in k}, f"{dump}.experts{rank}")
    dist.barrier()


def test_sft_source_rebuilds_fsdp_ep_snapshot(dsv4_dir, tmp_path):
    from tiny_dsv41_b200.train.sft_source import SFTCheckpointSource

    dump = tmp_path / "full.pt"
    run_gloo(_dsv4_fsdp, 2, dsv4_dir, tmp_path / "run", str(dump))
    source = SFTCheckpointSource(tmp_path / "run" / "checkpoint-00000001", dsv4_dir / "model")
    rebuilt = source.state_dict()
    dense = torch.load(dump)
    for name, value in dense.items():
        assert torch.equal(rebuilt[name].to(value.dtype), value), name
    for rank in range(2):
        for name, value in torch.load(f"{dump}.experts{rank}").items():
            half = value.shape[0]
            assert torch.equal(rebuilt[name][rank * half:(rank + 1) * half], value), name


def test_rl_policy_from_sft_snapshot(dsv4_dir, tmp_path):
    from tiny_dsv41_b200.rl.config import RLConfig
    from tiny_dsv41_b200.rl.family import load_model_config
    from tiny_dsv41_b200.rl.runtime import make_model

    run_gloo(_dsv4, 1, dsv4_dir, tmp_path / "sft", ["--steps", "1"])
    snapshot = tmp_path / "sft" / "checkpoint-00000001"
    saved = torch.load(snapshot / "rank-00000.pt", weights_only=False)
    cfg = RLConfig.from_dict(dict(rollout_engine="native-pytorch", initial_sft_checkpoint=str(snapshot)))
    model_dir = dsv4_dir / "model"
    policy = make_model(model_dir, load_model_config(model_dir), cfg, ("cpu",), False)
    params = dict(policy.backend.named_parameters())
    for name in ("model.layers.0.attention.q_a.weight", "model.layers.1.moe.routed.gate_up", "lm_head.weight"):
        assert torch.equal(params[name].detach(), saved["parameters"][name].to(params[name].dtype)), name
    rows = saved["engram_rows"]["tables"]["model.engram_tables.1.weight"]
    table = policy.backend.model.engram_tables["1"].weight
    assert torch.equal(table[rows["indices"]], rows["values"].to(table.dtype))


def test_dsv4_lora_sft_fp4_experts(dsv4_dir, tmp_path):
    out = tmp_path / "fp4"
    run_gloo(_dsv4, 1, dsv4_dir, out, ["--steps", "2", "--mode", "lora", "--fp4-experts", "--no-save"])
    losses, summary = _losses(out)
    assert len(losses) == 2 and all(l > 0 for l in losses)
    assert summary["eval_loss_after"] < summary["eval_loss_before"]
