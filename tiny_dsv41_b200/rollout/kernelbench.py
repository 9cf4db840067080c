"""Evaluation of model-written kernels (KernelBench-style tasks) with bounded concurrency.

The reference's rollout manager drives multi-turn CUDA-agent episodes whose candidates are
compiled and timed by pinned native harnesses (``rollout_manager/runner.py``,
``adapters/harnesses.py``, ``gpu_ownership.py``, ``host_memory.py``). This module is the
evaluation core of that loop, built for this library:

* a task (:class:`KernelCase`) is Python source that defines ``Model`` (the reference
  computation), ``get_inputs()`` and ``get_init_inputs()``; a candidate is Python source (usually
  the last fenced code block of a model response, :func:`extract_candidate`) that defines
  ``ModelNew`` with the same constructor and call signature;
* :func:`evaluate_candidate` runs one candidate in a spawned child process with a wall-clock
  limit, so a crash, a hang or a GPU fault in model-written code ends that child only. The child
  builds both models from the same seed (the candidate gets the reference's parameters where
  names match), checks outputs on several seeded input sets, then times both with device events
  (or the host clock on CPU) and reports a :class:`KernelVerdict`;
* :class:`KernelRunner` evaluates many (case, candidate) jobs: at most ``max_concurrency`` at a
  time, one job per device at a time (a device lease, so timings never share a GPU), a host-memory
  floor checked before each start, and a JSONL journal of queued / start / finish events plus one
  result record per job;
* :func:`kernel_reward` maps a verdict to a training reward (0 unless correct; then the clipped
  log2 speedup plus one), the quantity GRPO groups are built from;
* :func:`run_kernel_episode` is the multi-turn loop: the policy answers, the candidate is
  evaluated, the measured verdict goes back as the next user turn, and the last correct candidate
  is verified once more for the reward.
"""

from __future__ import annotations

import hashlib
import json
import math
import multiprocessing as mp
import re
import threading
import time
import traceback
from concurrent.futures import ThreadPoolExecutor
from dataclasses import asdict, dataclass, field
from pathlib import Path

STATUSES = ("correct", "incorrect", "error", "timeout")


@dataclass(frozen=True)
class KernelCase:
    case_id: str
    source: str  # defines Model, get_inputs(), get_init_inputs()
    atol: float = 1e-2
    rtol: float = 1e-2


@dataclass
class KernelVerdict:
    case_id: str
    candidate_sha256: str
    status: str
    detail: str = ""
    max_abs_error: float | None = None
    reference_ms: float | None = None
    candidate_ms: float | None = None
    speedup: float | None = None
    device: str = "cpu"
    seconds: float = 0.0
    extra: dict = field(default_factory=dict)


_FENCE = re.compile(r"```(?:python|py)?[ \t]*\n(.*?)```", re.DOTALL)


def extract_candidate(response: str) -> str | None:
    """The last fenced code block of a response that defines ``ModelNew`` (None when there is none)."""
    blocks = [b for b in _FENCE.findall(response) if re.search(r"^class\s+ModelNew\b", b, re.MULTILINE)]
    return blocks[-1] if blocks else None


def _sha(text: str) -> str:
    return hashlib.sha256(text.encode("utf-8")).hexdigest()


def _load(source: str, name: str, filename: str) -> dict:
    namespace: dict = {"__name__": name}
    exec(compile(source, filename, "exec"), namespace)  # noqa: S102 - evaluation runs in a child process
    return namespace


def _to(value, device):
    import torch

    if isinstance(value, torch.Tensor):
        return value.to(device)
    if isinstance(value, (list, tuple)):
        return type(value)(_to(v, device) for v in value)
    return value


def _time(fn, device, warmup: int, iters: int) -> float:
    import torch

    for _ in range(warmup):
        fn()
    if device.type == "cuda":
        torch.cuda.synchronize(device)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(iters):
            fn()
        end.record()
        torch.cuda.synchronize(device)
        return start.elapsed_time(end) / iters
    begin = time.perf_counter()
    for _ in range(iters):
        fn()
    return (time.perf_counter() - begin) * 1000.0 / iters


def _child(conn, case: KernelCase, candidate: str, device: str, trials: int, warmup: int, iters: int) -> None:
    """Runs in the spawned child: build, check, time; one verdict dict goes back over the pipe."""
    out = {"status": "error", "detail": ""}
    try:
        import torch

        dev = torch.device(device)
        if dev.type == "cuda":
            torch.cuda.set_device(dev)
        ref_ns = _load(case.source, "kernel_reference", f"<reference {case.case_id}>")
        try:
            cand_ns = _load(candidate, "kernel_candidate", "<candidate>")
            new_cls = cand_ns["ModelNew"]
        except Exception:  # the candidate does not even import
            out["detail"] = "candidate failed to load:\n" + traceback.format_exc(limit=3)
            conn.send(out)
            return
        init = ref_ns["get_init_inputs"]()
        torch.manual_seed(0)
        reference = ref_ns["Model"](*init).to(dev).eval()
        torch.manual_seed(0)
        model = new_cls(*init).to(dev).eval()
        # same parameters where the names and shapes agree
        theirs = dict(model.named_parameters())
        with torch.no_grad():
            for name, p in reference.named_parameters():
                if name in theirs and theirs[name].shape == p.shape:
                    theirs[name].copy_(p)
        worst = 0.0
        with torch.no_grad():
            for trial in range(trials):
                torch.manual_seed(1000 + trial)
                inputs = _to(ref_ns["get_inputs"](), dev)
                want = reference(*inputs)
                got = model(*inputs)
                want_list = [want] if isinstance(want, torch.Tensor) else list(want)
                got_list = [got] if isinstance(got, torch.Tensor) else list(got)
                for x, y in zip(got_list, want_list, strict=True):
                    if x.shape != y.shape:
                        raise ValueError(f"output shape {tuple(x.shape)} != reference {tuple(y.shape)}")
                    diff = (x.float() - y.float()).abs()
                    worst = max(worst, float(diff.max()) if diff.numel() else 0.0)
                    if not bool((diff <= case.atol + case.rtol * y.float().abs()).all()):
                        out.update(status="incorrect", max_abs_error=worst,
                                   detail=f"trial {trial}: outside atol {case.atol} / rtol {case.rtol}")
                        conn.send(out)
                        return
            torch.manual_seed(2000)
            inputs = _to(ref_ns["get_inputs"](), dev)
            ref_ms = _time(lambda: reference(*inputs), dev, warmup, iters)
            cand_ms = _time(lambda: model(*inputs), dev, warmup, iters)
        out.update(status="correct", max_abs_error=worst, reference_ms=ref_ms, candidate_ms=cand_ms,
                   speedup=ref_ms / cand_ms if cand_ms > 0 else None)
    except Exception:
        out.update(status="error", detail=traceback.format_exc(limit=4))
    conn.send(out)


def evaluate_candidate(case: KernelCase, candidate: str, *, device: str = "cpu", trials: int = 3, warmup: int = 3,
                       iters: int = 10, timeout: float = 120.0) -> KernelVerdict:
    """One candidate in a spawned child with a wall-clock limit (the child is killed past it)."""
    began = time.monotonic()
    verdict = KernelVerdict(case.case_id, _sha(candidate), "error", device=device)
    ctx = mp.get_context("spawn")
    parent, child = ctx.Pipe(duplex=False)
    proc = ctx.Process(target=_child, args=(child, case, candidate, device, trials, warmup, iters),
                       name=f"kernel-eval-{case.case_id}", daemon=True)
    proc.start()
    child.close()
    try:
        if parent.poll(timeout):
            result = parent.recv()
            for key, value in result.items():
                setattr(verdict, key, value)
        else:
            verdict.status, verdict.detail = "timeout", f"no verdict within {timeout:.0f} s"
    except EOFError:
        verdict.detail = f"evaluation process exited with code {proc.exitcode} before its verdict"
    finally:
        proc.join(timeout=1.0)
        if proc.is_alive():  # only this owned child is stopped
            proc.kill()
            proc.join()
        parent.close()
    verdict.seconds = time.monotonic() - began
    return verdict


def kernel_reward(verdict: KernelVerdict, *, max_log2_speedup: float = 3.0) -> float:
    """0 unless correct; then 1 + clip(log2(speedup), -1, max_log2_speedup), never below 0."""
    if verdict.status != "correct" or not verdict.speedup:
        return 0.0
    return max(0.0, 1.0 + min(max(math.log2(verdict.speedup), -1.0), max_log2_speedup))


class _DeviceLeases:
    """One evaluation per device at a time (timings never share a GPU); waits for a free device."""

    def __init__(self, devices) -> None:
        self.free = list(devices)
        self.cond = threading.Condition()

    def acquire(self) -> str:
        with self.cond:
            while not self.free:
                self.cond.wait()
            return self.free.pop(0)

    def release(self, device: str) -> None:
        with self.cond:
            self.free.append(device)
            self.cond.notify()


def available_host_bytes() -> int:
    import psutil

    return int(psutil.virtual_memory().available)


class KernelRunner:
    """Evaluates (case, candidate) jobs with at most ``max_concurrency`` in flight, one per device,
    starting a job only while the host has ``host_floor_bytes`` of memory available. Writes
    ``events.jsonl`` (queued / start / finish with monotonic ns) and ``results.jsonl`` under
    ``output_dir`` (created; an existing journal is never overwritten)."""

    def __init__(self, output_dir, *, devices=("cpu",), max_concurrency: int | None = None,
                 host_floor_bytes: int = 2 << 30, timeout: float = 120.0, trials: int = 3, warmup: int = 3,
                 iters: int = 10, memory_probe=available_host_bytes) -> None:
        self.output_dir = Path(output_dir)
        self.output_dir.mkdir(parents=True, exist_ok=True)
        self.events = (self.output_dir / "events.jsonl").open("x", encoding="utf-8")
        self.results = (self.output_dir / "results.jsonl").open("x", encoding="utf-8")
        self.leases = _DeviceLeases(devices)
        self.max_concurrency = max_concurrency or len(devices)
        self.host_floor_bytes = host_floor_bytes
        self.memory_probe = memory_probe
        self.options = {"timeout": timeout, "trials": trials, "warmup": warmup, "iters": iters}
        self.lock = threading.Lock()
        self.counts = {"queued": 0, "active": 0, "completed": 0}

    def _event(self, job: str, event: str, **details) -> None:
        with self.lock:
            if event == "queued":
                self.counts["queued"] += 1
            elif event == "start":
                self.counts["queued"] -= 1
                self.counts["active"] += 1
            elif event == "finish":
                self.counts["active"] -= 1
                self.counts["completed"] += 1
            record = {"monotonic_ns": time.monotonic_ns(), "job": job, "event": event, **details,
                      "counts": dict(self.counts)}
            self.events.write(json.dumps(record, sort_keys=True) + "\n")
            self.events.flush()

    def _wait_for_memory(self, job: str) -> None:
        waited = False
        while self.memory_probe() < self.host_floor_bytes:
            if not waited:
                self._event(job, "memory_wait", floor_bytes=self.host_floor_bytes)
                waited = True
            time.sleep(0.2)

    def _one(self, job: str, case: KernelCase, candidate: str) -> KernelVerdict:
        self._wait_for_memory(job)
        device = self.leases.acquire()
        self._event(job, "start", device=device)
        try:
            verdict = evaluate_candidate(case, candidate, device=device, **self.options)
        finally:
            self.leases.release(device)
        self._event(job, "finish", status=verdict.status)
        with self.lock:
            self.results.write(json.dumps({"job": job, **asdict(verdict), "reward": kernel_reward(verdict)},
                                          sort_keys=True) + "\n")
            self.results.flush()
        return verdict

    def evaluate(self, job: str, case: KernelCase, candidate: str) -> KernelVerdict:
        """One job through the same lease, memory floor and journal as :meth:`run`."""
        self._event(job, "queued")
        return self._one(job, case, candidate)

    def run(self, jobs) -> list[KernelVerdict]:
        """``jobs``: iterable of (job id, KernelCase, candidate source). Verdicts in job order."""
        jobs = list(jobs)
        for job, _, _ in jobs:
            self._event(job, "queued")
        with ThreadPoolExecutor(max_workers=self.max_concurrency, thread_name_prefix="kernel-eval") as pool:
            futures = [pool.submit(self._one, job, case, cand) for job, case, cand in jobs]
            return [f.result() for f in futures]

    def close(self) -> None:
        self.events.close()
        self.results.close()


def feedback_message(verdict: KernelVerdict) -> str:
    """The next user turn of a feedback episode: the measured verdict of the previous candidate."""
    measured = {"status": verdict.status, "detail": verdict.detail[:2000], "max_abs_error": verdict.max_abs_error,
                "reference_ms": verdict.reference_ms, "candidate_ms": verdict.candidate_ms,
                "speedup": verdict.speedup}
    return ("Your previous candidate was compiled, checked and timed. Measured result:\n" + json.dumps(measured) +
            "\nReply with a complete improved candidate: one fenced Python block defining ModelNew with the "
            "same constructor arguments, forward signature and output shapes as Model.")


def run_kernel_episode(case: KernelCase, generate, runner: KernelRunner, prompt, *, turns: int = 2,
                       job: str | None = None) -> dict:
    """A multi-turn kernel episode (the reference's ``--turns 2`` mode of ``rollout_manager/runner.py``).

    ``generate(messages) -> str`` is the policy (chat messages in, assistant text out). Each turn's
    candidate is evaluated through ``runner``; from the second turn on, the conversation carries the
    previous reply and its measured verdict (:func:`feedback_message`). The last correct turn is
    selected and verified once more with a fresh evaluation, whose verdict gives the reward (0 when
    no turn was correct). Returns the episode record: per-turn candidate digests and verdicts, the
    selected turn, the verification verdict and the reward."""
    if turns < 1:
        raise ValueError("an episode needs at least one turn")
    job = job or case.case_id
    messages = list(prompt) if isinstance(prompt, (list, tuple)) else [{"role": "user", "content": str(prompt)}]
    record = {"job": job, "case_id": case.case_id, "turns": [], "selected_turn": None, "verification": None,
              "reward": 0.0}
    selected = None
    for index in range(turns):
        reply = generate(list(messages))
        candidate = extract_candidate(reply) or ""
        verdict = runner.evaluate(f"{job}-t{index + 1}", case, candidate)
        record["turns"].append({"turn": index + 1, "candidate_sha256": verdict.candidate_sha256,
                                "extracted": bool(candidate), "verdict": asdict(verdict)})
        if verdict.status == "correct":
            selected = (index + 1, candidate)
        if index + 1 < turns:
            messages += [{"role": "assistant", "content": reply}, {"role": "user", "content": feedback_message(verdict)}]
    if selected is not None:
        record["selected_turn"] = selected[0]
        final = runner.evaluate(f"{job}-verify", case, selected[1])
        record["verification"] = asdict(final)
        record["reward"] = kernel_reward(final)
    return record


QUALIFICATION_FORMAT = "kernel-reference-qualification-v1"


def self_candidate(case: KernelCase) -> str:
    """The task's own reference as a candidate (``ModelNew`` is ``Model``)."""
    return case.source + "\n\nclass ModelNew(Model):\n    pass\n"


def _cases_digest(cases) -> str:
    return _sha(json.dumps(sorted((c.case_id, _sha(c.source)) for c in cases)))


def qualify_cases(cases, runner: KernelRunner, *, job_prefix: str = "qualify") -> dict:
    """Score eligibility of each task, decided by running its reference through the same harness as
    a candidate (the role of the reference's ``reference_qualification.py``): a task whose reference
    does not pass against itself (it errors, times out, or its outputs are not reproducible within
    the task's tolerance, e.g. randomness inside ``forward``) can never be scored fairly and is
    excluded. The catalog binds each decision to the task source digest."""
    cases = list(cases)
    verdicts = runner.run([(f"{job_prefix}-{c.case_id}", c, self_candidate(c)) for c in cases])
    tasks = {}
    for case, verdict in zip(cases, verdicts):
        eligible = verdict.status == "correct"
        reason = None if eligible else f"reference against itself: {verdict.status}: {verdict.detail[:300]}"
        tasks[case.case_id] = {"source_sha256": _sha(case.source), "score_eligible": eligible, "reason": reason,
                               "max_abs_error": verdict.max_abs_error}
    return {"format": QUALIFICATION_FORMAT, "cases_sha256": _cases_digest(cases), "tasks": tasks}


def check_qualification(catalog: dict, cases) -> dict[str, bool]:
    """Eligibility per case id from a catalog of :func:`qualify_cases`, refusing one made for other
    task sources or another set of tasks."""
    cases = list(cases)
    if catalog.get("format") != QUALIFICATION_FORMAT or catalog.get("cases_sha256") != _cases_digest(cases):
        raise ValueError("the qualification catalog was made for another set of tasks")
    tasks = catalog["tasks"]
    if set(tasks) != {c.case_id for c in cases}:
        raise ValueError("the qualification catalog covers other tasks")
    out = {}
    for case in cases:
        item = tasks[case.case_id]
        if item["source_sha256"] != _sha(case.source) or type(item["score_eligible"]) is not bool:
            raise ValueError(f"qualification of {case.case_id} does not match its source")
        out[case.case_id] = item["score_eligible"]
    return out


def load_cases(directory) -> list[KernelCase]:
    """Every ``*.py`` file of a directory as a case named after the file (sorted)."""
    return [KernelCase(p.stem, p.read_text(encoding="utf-8")) for p in sorted(Path(directory).glob("*.py"))]


def main(argv=None) -> None:
    import argparse

    parser = argparse.ArgumentParser(description="Evaluate model-written kernels against reference tasks")
    parser.add_argument("--cases", required=True, help="directory of task files (Model, get_inputs, get_init_inputs)")
    parser.add_argument("--responses", required=True,
                        help="JSONL of {case_id, response} (model output with a fenced ModelNew block)")
    parser.add_argument("--output-dir", required=True)
    parser.add_argument("--devices", default="cpu", help="comma-separated, e.g. cuda:0,cuda:1")
    parser.add_argument("--timeout", type=float, default=120.0)
    args = parser.parse_args(argv)
    cases = {c.case_id: c for c in load_cases(args.cases)}
    jobs = []
    for n, line in enumerate(Path(args.responses).read_text(encoding="utf-8").splitlines()):
        if not line.strip():
            continue
        row = json.loads(line)
        code = extract_candidate(row["response"]) or ""
        jobs.append((f"{row['case_id']}#{n}", cases[row["case_id"]], code))
    runner = KernelRunner(args.output_dir, devices=args.devices.split(","), timeout=args.timeout)
    try:
        verdicts = runner.run(jobs)
    finally:
        runner.close()
    summary = {s: sum(v.status == s for v in verdicts) for s in STATUSES}
    print(json.dumps({"jobs": len(verdicts), **summary}), flush=True)


if __name__ == "__main__":
    main()


__all__ = ["KernelCase", "KernelRunner", "KernelVerdict", "evaluate_candidate", "extract_candidate",
           "check_qualification", "feedback_message", "kernel_reward", "load_cases", "qualify_cases",
           "run_kernel_episode", "self_candidate"]
