"""Kernel-evaluation runner (rollout/kernelbench.py) on CPU: correct, incorrect, broken and hanging
candidates, reward mapping, device leases and the journal."""

import json

from tiny_dsv41_b200.rollout.kernelbench import (KernelCase, KernelRunner, evaluate_candidate, extract_candidate,
                                                 kernel_reward)

TASK = '''
import torch
from torch import nn

class Model(nn.Module):
    def __init__(self, n):
        super().__init__()
        self.proj = nn.Linear(n, n)

    def forward(self, x):
        return torch.relu(self.proj(x))

def get_inputs():
    return [torch.randn(8, 16)]

def get_init_inputs():
    return [16]
'''

GOOD = '''
import torch
from torch import nn

class ModelNew(nn.Module):
    def __init__(self, n):
        super().__init__()
        self.proj = nn.Linear(n, n)

    def forward(self, x):
        return torch.clamp_min(x @ self.proj.weight.t() + self.proj.bias, 0.0)
'''

WRONG = GOOD.replace("clamp_min(", "clamp_min(0.5 + ")
BROKEN = "class ModelNew(:\n    pass\n"
HANGS = GOOD.replace("return torch.clamp_min", "while True:\n            pass\n        return torch.clamp_min")


def test_extract_candidate_takes_last_modelnew_block():
    response = "text\n```python\nx = 1\n```\nmore\n```python\nclass ModelNew:\n    pass\n```\n"
    assert extract_candidate(response).startswith("class ModelNew")
    assert extract_candidate("no code here") is None


def test_verdicts_and_rewards():
    case = KernelCase("relu_linear", TASK)
    good = evaluate_candidate(case, GOOD, iters=3, warmup=1, timeout=60)
    assert good.status == "correct" and good.max_abs_error < 1e-4 and good.speedup > 0, good
    assert kernel_reward(good) > 0
    wrong = evaluate_candidate(case, WRONG, iters=3, warmup=1, timeout=60)
    assert wrong.status == "incorrect" and kernel_reward(wrong) == 0.0, wrong
    broken = evaluate_candidate(case, BROKEN, timeout=60)
    assert broken.status == "error" and "failed to load" in broken.detail, broken
    hung = evaluate_candidate(case, HANGS, timeout=20)
    assert hung.status == "timeout" and kernel_reward(hung) == 0.0, hung


def test_runner_leases_and_journal(tmp_path):
    case = KernelCase("relu_linear", TASK)
    probes = iter([0, 0] + [1 << 40] * 100)  # the first start waits for host memory
    runner = KernelRunner(tmp_path / "run", devices=("cpu", "cpu"), timeout=60, iters=2, warmup=1,
                          host_floor_bytes=1, memory_probe=lambda: next(probes))
    try:
        verdicts = runner.run([("a", case, GOOD), ("b", case, WRONG), ("c", case, GOOD)])
    finally:
        runner.close()
    assert [v.status for v in verdicts] == ["correct", "incorrect", "correct"]
    events = [json.loads(line) for line in (tmp_path / "run" / "events.jsonl").read_text().splitlines()]
    assert [e["event"] for e in events].count("finish") == 3
    assert any(e["event"] == "memory_wait" for e in events)
    assert max(e["counts"]["active"] for e in events) <= 2
    assert events[-1]["counts"] == {"queued": 0, "active": 0, "completed": 3}
    rows = [json.loads(line) for line in (tmp_path / "run" / "results.jsonl").read_text().splitlines()]
    assert sorted(r["job"] for r in rows) == ["a", "b", "c"]
