"""GRPO learner: CPU parity with the reference learner step, and the local run end to end.

The parity case is the CPU GRPO plumbing configuration: the tiny random-init DSV4.1 model of
``examples/tiny-dsv41``, fp32, seed 0, 8 prompts of 32 uniform-random token ids, G = 4 samples
of 16 new tokens at temperature 1.0, reward = fraction of generated tokens equal to a fixed id,
two learner steps.
"""

import json
import random
from pathlib import Path

import pytest
import torch

from tests.ref_oracle import import_reference, reference_available
from tiny_dsv41_b200.rl.config import RLConfig
from tiny_dsv41_b200.rl.data import PromptRecord
from tiny_dsv41_b200.rl.family import build_policy, load_model_config
from tiny_dsv41_b200.rl.rollout import generate_group
from tiny_dsv41_b200.rl.runtime import train_groups

ROOT = Path(__file__).resolve().parents[1]
MODEL = ROOT / "examples" / "tiny-dsv41"
TARGET = 7


def _reward(record, response):
    return sum(t == TARGET for t in response) / len(response)


def _records():
    rng = random.Random(0)
    return [PromptRecord([rng.randrange(32) for _ in range(32)]) for _ in range(8)]


def _config(**kw):
    values = dict(group_size=4, max_new_tokens=16, temperature=1.0, rollout_engine="native-pytorch", seed=0,
                  learning_rate=1e-3)
    values.update(kw)
    return RLConfig.from_dict(values)


@pytest.mark.skipif(not reference_available(), reason="reference package not installed")
def test_train_groups_parity_with_reference():
    import_reference()
    from dsv41_train.models.dsv4.model import DeepSeekV41ForCausalLM as RefModel
    from dsv41_train.rl.config import RLConfig as RefRLConfig
    from dsv41_train.rl.policy import DSV41Config as RefConfig, DSV41Policy as RefPolicy
    from dsv41_train.rl.rollout import RolloutGroup as RefGroup, Sample as RefSample
    from dsv41_train.rl.runtime import train_groups as ref_train_groups

    torch.manual_seed(0)
    cfg = _config()
    model_config = load_model_config(MODEL)
    ours = build_policy(MODEL, model_config, random_init=True, devices=("cpu",), dtype=torch.float32)
    ref_backend = RefModel(RefConfig.from_model_dir(MODEL))
    missing, unexpected = ref_backend.load_state_dict(ours.backend.state_dict(), strict=False)
    assert not missing and not unexpected, (missing, unexpected)
    ref = RefPolicy(ref_backend).to_training_devices(("cpu",), torch.float32)
    ref_cfg = RefRLConfig.from_dict(dict(group_size=4, max_new_tokens=16, temperature=1.0, seed=0,
                                         learning_rate=1e-3, rollout_engine="native-pytorch"))
    opt_a = torch.optim.AdamW([p for p in ours.parameters() if p.requires_grad], lr=1e-3, weight_decay=0.0,
                              foreach=False)
    opt_b = torch.optim.AdamW([p for p in ref.parameters() if p.requires_grad], lr=1e-3, weight_decay=0.0,
                              foreach=False)
    names_a = [n.removeprefix("backend.") for n, p in ours.named_parameters() if p.requires_grad]
    names_b = [n.removeprefix("backend.") for n, p in ref.named_parameters() if p.requires_grad]
    assert names_a == names_b
    grads = {"a": [], "b": []}
    trainable_a = [p for p in ours.parameters() if p.requires_grad]
    trainable_b = [p for p in ref.parameters() if p.requires_grad]
    opt_a.register_step_pre_hook(lambda *_: grads["a"].append([p.grad.clone() for p in trainable_a]))
    opt_b.register_step_pre_hook(lambda *_: grads["b"].append([p.grad.clone() for p in trainable_b]))
    generator = torch.Generator().manual_seed(0)
    records = _records()
    for step in range(2):
        groups = [generate_group(ours, r, 4, 16, 1.0, eos_token_id=None, policy_version=step, group_id=i,
                                 generator=generator, reward_fn=_reward) for i, r in enumerate(records)]
        ref_groups = [RefGroup([RefSample(s.prompt_ids, s.response_ids, s.behavior_log_probs, s.reward,
                                          s.policy_version, s.finish_reason, s.stop_token_count)
                                for s in g.samples], g.group_id, g.policy_version) for g in groups]
        a = train_groups(ours, None, opt_a, groups, cfg)
        b = ref_train_groups(ref, None, opt_b, ref_groups, ref_cfg)
        for key in ("loss", "policy_loss", "reward_mean", "grad_norm"):
            assert a[key] == pytest.approx(b[key], rel=1e-4, abs=1e-6), (step, key, a[key], b[key])
        # the gradients the optimizer sees, parameter by parameter, relative to each one's largest entry
        for name, ga, gb in zip(names_a, grads["a"][step], grads["b"][step]):
            scale = gb.abs().max().item()
            assert (ga - gb).abs().max().item() <= 1e-4 * scale + 1e-9, (step, name, scale)
        # Adam divides by sqrt(v): where a gradient entry is ~0 its rounding differences reach the update at
        # up to lr scale, so the updated parameters agree to the learning rate. The next step then starts
        # both sides from our state (parameters and moments), so its gradients are compared as tightly.
        with torch.no_grad():
            for name, p, q in zip(names_a, trainable_a, trainable_b):
                assert (p - q).abs().max().item() < 1e-3, (step, name, (p - q).abs().max().item())
                q.copy_(p)
                for key, value in opt_a.state[p].items():
                    opt_b.state[q][key].copy_(value)


def test_local_grpo_run_and_resume(tmp_path):
    from tiny_dsv41_b200.rl.runtime import run_training

    data = tmp_path / "data.jsonl"
    with data.open("w") as f:
        for r in _records()[:4]:
            f.write(json.dumps({"prompt_ids": r.prompt_ids[:8], "target_ids": [TARGET] * 3}) + "\n")
    cfg = dict(max_steps=2, group_size=2, max_new_tokens=3, rollout_engine="native-pytorch", seed=0,
               output_dir=str(tmp_path / "out"), worker_timeout_seconds=300)
    last = run_training(model_dir=MODEL, data_path=data, config=RLConfig.from_dict(cfg), random_init=True)
    out = tmp_path / "out"
    assert last == out / "step-00000002.pt"
    assert len(list((out / "policies").glob("policy-*.pt"))) == 3
    rows = [json.loads(line) for line in (out / "metrics.jsonl").read_text().splitlines()]
    assert [r["step"] for r in rows] == [1, 2] and all(r["optimizer_step_applied"] for r in rows)
    stages = {json.loads(line)["stage"] for line in (out / "learner-stage-timings.jsonl").read_text().splitlines()}
    assert {"model_startup", "train_groups", "policy_publish", "checkpoint_write", "actor_activation"} <= stages
    resumed = run_training(model_dir=MODEL, data_path=data, config=RLConfig.from_dict({**cfg, "max_steps": 3}),
                           random_init=True, resume=last)
    assert resumed == out / "step-00000003.pt"
    with pytest.raises(FileExistsError):
        run_training(model_dir=MODEL, data_path=data, config=RLConfig.from_dict(cfg), random_init=True)
    # standalone sampling and evaluation from the saved checkpoint
    from tiny_dsv41_b200.rl.evaluate import main as evaluate_main
    from tiny_dsv41_b200.rl.sample import sample_checkpoint

    result = sample_checkpoint(model_dir=MODEL, checkpoint=resumed, prompt_ids=[1, 2, 3], seed=5)
    assert result["policy_version"] == 3 and len(result["response_ids"]) == 3
    again = sample_checkpoint(model_dir=MODEL, checkpoint=resumed, prompt_ids=[1, 2, 3], seed=5)
    assert again["response_ids"] == result["response_ids"]
    evaluate_main(["--model-dir", str(MODEL), "--checkpoint", str(resumed), "--data", str(data), "--output-dir",
                   str(tmp_path / "eval")])
    metrics = json.loads((tmp_path / "eval" / "eval-metrics.jsonl").read_text().splitlines()[-1])
    assert metrics["step"] == 3 and metrics["prompts"] == 4


def test_qwen_head_example_runs_and_checkpoints(tmp_path):
    """The shipped tiny Qwen3-MoE fixture and lm_head-only config train through the manager and
    close it cleanly (its recovery snapshot carries the sampler RNG state)."""
    import json
    import subprocess
    import sys

    root = Path(__file__).resolve().parents[1]
    config = json.loads((root / "examples/rl/qwen-head.json").read_text())
    config.update(max_steps=2, output_dir=str(tmp_path / "out"))
    cfg_path = tmp_path / "qwen-head.json"
    cfg_path.write_text(json.dumps(config))
    proc = subprocess.run([sys.executable, "-m", "tiny_dsv41_b200.rl.train", "--model-dir",
                           str(root / "examples/tiny-qwen3"), "--data", str(root / "examples/rl/prompts.jsonl"),
                           "--config", str(cfg_path), "--random-init"],
                          cwd=root, capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stderr[-2000:]
    state = torch.load(tmp_path / "out" / "step-00000002.pt", weights_only=False)
    assert state["step"] == 2 and state["rollout_rng_state"].dtype == torch.uint8


def test_admit_packet_drops_exclusions_and_stale_groups(tmp_path):
    """Rollout packets the learner cannot train on are committed as dropped; provider exclusions
    are also logged to excluded-groups.jsonl."""
    import json
    from types import SimpleNamespace

    from tiny_dsv41_b200.rl.runtime import admit_packet

    class Manager:
        def __init__(self):
            self.dropped = []

        def commit(self, consumed_group_ids=(), dropped_group_ids=()):
            self.dropped += list(dropped_group_ids)

    config = SimpleNamespace(max_policy_lag=1, group_size=2)
    manager = Manager()
    assert admit_packet({"exclusion": {"group_id": 5, "reasons": ["bad"]}, "group_id": 5}, 3, config, manager,
                        tmp_path) is None
    stale = SimpleNamespace(group_id=6, policy_version=1, samples=[0, 1])
    assert admit_packet({"group": stale}, 3, config, manager, tmp_path) is None
    fresh = SimpleNamespace(group_id=7, policy_version=2, samples=[0, 1])
    assert admit_packet({"group": fresh}, 3, config, manager, tmp_path) == (fresh, 1)
    assert manager.dropped == [5, 6]
    logged = [json.loads(line) for line in (tmp_path / "excluded-groups.jsonl").read_text().splitlines()]
    assert logged == [{"group_id": 5, "reasons": ["bad"]}]
    with pytest.raises(ValueError):
        admit_packet({"group": SimpleNamespace(group_id=8, policy_version=3, samples=[0])}, 3, config, manager,
                     tmp_path)
