"""The original module paths (``dsv41_train.*``, ``rollout_manager.*``) resolve to this library's
modules when the compatibility packages are installed, and ``python -m dsv41_train.rl.train``
runs this library's GRPO runtime end to end. Run in subprocesses so that the test process keeps
importing the original package for the parity tests."""

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
ENV = {**os.environ, "PYTHONPATH": os.pathsep.join([str(ROOT / "compat"), str(ROOT)])}


def _run(args, **kw):
    return subprocess.run([sys.executable, *args], cwd=ROOT, env=ENV, capture_output=True, text=True, timeout=600,
                          **kw)


def test_library_module_paths_alias_this_library():
    code = (
        "import dsv41_train.models.qwen as a, tiny_dsv41_b200.models.qwen as b; assert a is b\n"
        "import dsv41_train.rl.algorithm as c, tiny_dsv41_b200.rl.algorithm as d; assert c is d\n"
        "from dsv41_train.cp import ContextParallel, pack_sequences\n"
        "from dsv41_train.lora import inject_lora\n"
        "from dsv41_train.optim import install_sgd_in_backward\n"
        "from rollout_manager.training import TrainingGroup\n"
        "from rollout_manager.backends.vllm_lora_transport import pack_update\n"
        "print(ContextParallel.__module__, TrainingGroup.__module__)\n"
    )
    proc = _run(["-c", code])
    assert proc.returncode == 0, proc.stderr[-2000:]
    assert proc.stdout.split() == ["tiny_dsv41_b200.parallel.cp", "tiny_dsv41_b200.rollout.training"]


def test_rl_cli_runs_under_the_original_module_path(tmp_path):
    data = tmp_path / "prompts.jsonl"
    data.write_text("".join(json.dumps({"prompt_ids": [1, 2, 3, 4], "target_ids": [5]}) + "\n" for _ in range(2)))
    config = tmp_path / "rl.json"
    config.write_text(json.dumps(dict(max_steps=1, group_size=2, max_new_tokens=2, rollout_engine="native-pytorch",
                                      seed=0, output_dir=str(tmp_path / "out"))))
    proc = _run(["-m", "dsv41_train.rl.train", "--model-dir", str(ROOT / "examples" / "tiny-dsv41"), "--data",
                 str(data), "--config", str(config), "--random-init"])
    assert proc.returncode == 0, proc.stderr[-2000:]
    assert (tmp_path / "out" / "step-00000001.pt").exists()
    for module in ("dsv41_train.rl.sample", "dsv41_train.rl.evaluate", "dsv41_train.rl.distributed_grpo",
                   "rollout_manager"):
        help_proc = _run(["-m", module, "--help"])
        assert help_proc.returncode == 0, (module, help_proc.stderr[-1000:])
