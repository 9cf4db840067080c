"""Kernel-evaluation runner (rollout/kernelbench.py) on CPU: correct, incorrect, broken and hanging
candidates, reward mapping, device leases and the journal."""

import json
import math

from tiny_dsv41_b200.rollout.kernelbench import (KernelCase, KernelRunner, KernelVerdict, evaluate_candidate,
                                                 extract_candidate, kernel_reward)

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
    # a correct candidate's reward follows its measured speedup (CPU timings of a shared host are
    # noise, so the value itself is not asserted)
    assert kernel_reward(good) == max(0.0, 1.0 + min(max(math.log2(good.speedup), -1.0), 3.0))
    fast = KernelVerdict("relu_linear", "x", "correct", speedup=2.0)
    assert kernel_reward(fast) == 2.0 and kernel_reward(KernelVerdict("relu_linear", "x", "correct", speedup=64.0)) == 4.0
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


def test_feedback_episode_selects_the_last_correct_turn(tmp_path):
    """Turn 1 answers wrongly, turn 2 sees the measured verdict of turn 1 and answers correctly; the
    correct turn is verified once more and gives the reward."""
    from tiny_dsv41_b200.rollout.kernelbench import run_kernel_episode

    case = KernelCase("relu_linear", TASK)
    seen = []

    def policy(messages):
        seen.append(messages)
        code = WRONG if len(messages) == 1 else GOOD
        return "Here is my kernel.\n```python\n" + code + "```\n"

    runner = KernelRunner(tmp_path / "ep", devices=("cpu",), timeout=60, trials=2, warmup=1, iters=2)
    try:
        record = run_kernel_episode(case, policy, runner, "Write ModelNew for this task.", turns=2, job="ep0")
    finally:
        runner.close()
    assert [t["verdict"]["status"] for t in record["turns"]] == ["incorrect", "correct"], record
    assert record["selected_turn"] == 2 and record["verification"]["status"] == "correct"
    # the reward is the verification's (its speedup on a shared CPU is noise, so only its form is checked)
    speedup = record["verification"]["speedup"]
    assert speedup and record["reward"] == max(0.0, 1.0 + min(max(math.log2(speedup), -1.0), 3.0))
    # the second request carries the first reply and its measured verdict
    assert len(seen[1]) == 3 and seen[1][1]["role"] == "assistant" and '"status": "incorrect"' in seen[1][2]["content"]
    events = [json.loads(line) for line in (tmp_path / "ep" / "events.jsonl").read_text().splitlines()]
    assert {e["job"] for e in events} == {"ep0-t1", "ep0-t2", "ep0-verify"}


def test_feedback_episode_without_a_correct_turn_has_no_reward(tmp_path):
    from tiny_dsv41_b200.rollout.kernelbench import run_kernel_episode

    runner = KernelRunner(tmp_path / "ep", devices=("cpu",), timeout=60, trials=1, warmup=1, iters=1)
    try:
        record = run_kernel_episode(KernelCase("relu_linear", TASK), lambda m: "no code here", runner, "task",
                                    turns=2)
    finally:
        runner.close()
    assert record["selected_turn"] is None and record["reward"] == 0.0 and record["verification"] is None
    assert all(not t["extracted"] for t in record["turns"])


NOISY = TASK.replace("return torch.relu(self.proj(x))", "return torch.relu(self.proj(x)) + torch.rand_like(x)")


def test_reference_qualification_excludes_irreproducible_tasks(tmp_path):
    from tiny_dsv41_b200.rollout.kernelbench import check_qualification, qualify_cases

    cases = [KernelCase("stable", TASK), KernelCase("noisy", NOISY)]
    runner = KernelRunner(tmp_path / "q", devices=("cpu",), timeout=60, trials=2, warmup=1, iters=1)
    try:
        catalog = qualify_cases(cases, runner)
    finally:
        runner.close()
    assert catalog["tasks"]["stable"]["score_eligible"] is True
    assert catalog["tasks"]["noisy"]["score_eligible"] is False and "incorrect" in catalog["tasks"]["noisy"]["reason"]
    assert check_qualification(json.loads(json.dumps(catalog)), cases) == {"stable": True, "noisy": False}
    edited = [KernelCase("stable", TASK + "\n# edited\n"), cases[1]]
    try:
        check_qualification(catalog, edited)
    except ValueError:
        pass
    else:
        raise AssertionError("a catalog of other task sources was accepted")
