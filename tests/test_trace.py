"""Opt-in distributed trace points and NVTX ranges."""

import json

from tiny_dsv41_b200.utils import trace


def test_trace_points_to_directory(tmp_path, monkeypatch):
    monkeypatch.setenv("RANK", "3")
    trace.set_tracing(distributed=False, directory=str(tmp_path))
    try:
        trace.trace_point("step_begin", step=7)
        trace.trace_point("step_end", step=7, loss=1.5)
    finally:
        trace.set_tracing(directory="")
    rows = [json.loads(line) for line in (tmp_path / "trace-rank-3.jsonl").read_text().splitlines()]
    assert [r["event"] for r in rows] == ["step_begin", "step_end"]
    assert rows[1]["rank"] == 3 and rows[1]["loss"] == 1.5 and rows[0]["monotonic"] <= rows[1]["monotonic"]


def test_disabled_trace_and_nvtx_are_no_ops(capsys):
    trace.set_tracing(distributed=False, nvtx=False, directory="")
    trace.trace_point("ignored")
    with trace.nvtx_range("phase"):
        pass
    assert capsys.readouterr().err == ""


def test_stderr_trace(capsys):
    trace.set_tracing(distributed=True)
    try:
        trace.trace_point("loaded", seconds=0.25)
    finally:
        trace.set_tracing(distributed=False)
    line = capsys.readouterr().err.strip()
    assert json.loads(line)["event"] == "loaded"
