"""Terminal-Bench-style episodes (rollout/terminal.py) on the host: scripted agents, the task's
own verification, timeouts, sealed evidence and the coordinator backend interface."""

import asyncio
import json
from pathlib import Path

import pytest

from tiny_dsv41_b200.rollout.contracts import EpisodeIdentity, EpisodePlan, ResourceRequirements, TaskSpec
from tiny_dsv41_b200.rollout.coordinator import Coordinator
from tiny_dsv41_b200.rollout.terminal import SandboxLimits, TerminalBackend, run_episode, verify_evidence


def _task(root: Path) -> Path:
    task = root / "hello"
    (task / "workspace").mkdir(parents=True)
    (task / "tests").mkdir()
    (task / "instruction.md").write_text("Write the word hi into hello.txt.\n")
    (task / "workspace" / "README").write_text("seed file\n")
    (task / "tests" / "run.sh").write_text('test "$(cat "$1/hello.txt" 2>/dev/null)" = hi\n')
    return task


def _scripted(*commands):
    def agent(instruction, transcript):
        return commands[len(transcript)] if len(transcript) < len(commands) else None
    return agent


def test_episode_outcomes_and_evidence(tmp_path):
    task = _task(tmp_path)
    good = run_episode(task, _scripted("ls", "echo hi > hello.txt"), tmp_path / "ev-good")
    assert good["passed"] and good["reward"] == 1.0 and good["commands"] == 2
    manifest = verify_evidence(tmp_path / "ev-good")
    transcript = json.loads((tmp_path / "ev-good" / "transcript.json").read_text())
    assert "README" in transcript[0]["output"] and manifest["workspace_sha256"]
    bad = run_episode(task, _scripted("echo no > hello.txt"), tmp_path / "ev-bad")
    assert not bad["passed"] and bad["reward"] == 0.0
    hung = run_episode(task, _scripted("sleep 30"), tmp_path / "ev-hung", SandboxLimits(command_seconds=1))
    assert not hung["passed"]
    assert json.loads((tmp_path / "ev-hung" / "transcript.json").read_text())[0]["timed_out"]
    # the agent cannot reach the tests: they are copied after its last command, outside its tree
    sneaky = run_episode(task, _scripted("mkdir -p ../tests && echo 'exit 0' > ../tests/run.sh"), tmp_path / "ev-s")
    assert not sneaky["passed"]
    (tmp_path / "ev-good" / "transcript.json").write_text("[]")
    with pytest.raises(ValueError):
        verify_evidence(tmp_path / "ev-good")


def test_backend_through_the_coordinator(tmp_path):
    task = _task(tmp_path)
    spec = TaskSpec("terminal-bench", "hello", "0" * 64, {"task_path": str(task)}, ResourceRequirements("cpu"))
    plans = [EpisodePlan(EpisodeIdentity("run", "terminal-bench", "hello", "g0", i), spec) for i in range(3)]
    agents = {0: _scripted("echo hi > hello.txt"), 1: _scripted("echo nope > hello.txt"),
              2: _scripted("printf hi > hello.txt")}
    backend = TerminalBackend(lambda plan: agents[plan.identity.sample_index], tmp_path / "evidence")

    async def scenario():
        coord = Coordinator({"terminal-bench": backend}, max_workers=2)
        await coord.open_stream(max_pending=3)
        results = await coord.execute_stream_group(plans, sequence=0)
        await coord.close_stream()
        return results

    results = asyncio.run(scenario())
    assert [r.native_outcome["passed"] for r in results] == [True, False, True]
    assert all(r.score_eligible and r.cleanup_state == "clean" for r in results)
    for r in results:
        verify_evidence(Path(r.native_artifacts["evidence"]))
