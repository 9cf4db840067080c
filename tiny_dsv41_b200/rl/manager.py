"""Rollout manager: GRPO groups sampled by a spawned child process with the active policy.

Learner-facing contract (the one ``dsv41_train/rl/manager.py:17-357`` defines, and the recovery
snapshot stored in RL checkpoints):

* ``start()`` spawns the child; it builds its own policy on the rollout devices, activates the
  initial policy artifact and replies with the activation receipt ``{version, digest, lineage}``.
* ``get(timeout)`` hands over the oldest undelivered group packet, or raises ``queue.Empty``.
* ``pause()`` stops admission at the next group boundary and returns the recovery snapshot.
* ``commit(consumed, dropped)`` retires delivered groups; they must be the oldest ones, in order.
* ``activate(artifact)`` (paused) loads a newly published artifact and returns its receipt.
* ``resume()`` re-opens admission; ``evaluate(records, step=...)`` (paused) scores the active
  policy; ``close()`` drains the child and returns the final snapshot.

Structure here: the child keeps its groups in a :class:`_Mailbox` (cursor, committed high-water
mark, bounded slots) and answers requests through a table of handlers, sampling one group between
request polls whenever the mailbox has room; the learner talks to it through a :class:`_Link`
(numbered requests, replies that must echo the number, a deadline, and the child's traceback on
failure). The mailbox holds at most ``queue_capacity + groups_per_step`` groups.
"""

from __future__ import annotations

import multiprocessing as mp
import queue
import time
import traceback
import uuid
from collections import OrderedDict
from dataclasses import asdict
from pathlib import Path

import torch

SNAPSHOT_SCHEMA = 1


# ---------------------------------------------------------------------------------------------
# wire encoding of packets (dataclasses do not cross the pipe as such)
# ---------------------------------------------------------------------------------------------
def _pack(packet: dict) -> dict:
    return {**packet, "group": asdict(packet["group"])}


def _unpack(packet: dict) -> dict:
    from .rollout import RolloutGroup, Sample

    group = packet["group"]
    samples = [Sample(**fields) for fields in group["samples"]]
    return {**packet, "group": RolloutGroup(samples, group["group_id"], group["policy_version"])}


class _Mailbox:
    """Sampled groups between admission and commit: ids ``[highwater, next_id)`` without gaps."""

    def __init__(self, bound: int, next_id: int, highwater: int, dropped: int) -> None:
        self.bound = bound
        self.next_id = next_id
        self.highwater = highwater
        self.dropped = dropped
        self.slots: OrderedDict[int, list] = OrderedDict()  # id -> [packet, delivered]

    @classmethod
    def restore(cls, recovery: dict, bound: int, default_next: int) -> "_Mailbox":
        next_id = recovery.get("next_group_id", default_next)
        box = cls(bound, next_id, recovery.get("committed_highwater", next_id), recovery.get("dropped_groups", 0))
        for encoded in recovery.get("pending_packets", []):
            packet = _unpack(encoded)
            gid = packet["group"].group_id
            if gid in box.slots or not box.highwater <= gid < box.next_id:
                raise ValueError("invalid or duplicate restored group cursor")
            box.slots[gid] = [packet, False]
        box.slots = OrderedDict(sorted(box.slots.items()))
        if len(box.slots) > bound or list(box.slots) != list(range(box.highwater, box.next_id)):
            raise ValueError("restored mailbox exceeds capacity or has a cursor gap")
        return box

    def waiting(self) -> int:
        return sum(1 for _, delivered in self.slots.values() if not delivered)

    def has_room(self, queue_capacity: int) -> bool:
        return len(self.slots) < self.bound and self.waiting() < queue_capacity

    def reserve(self) -> int:
        gid, self.next_id = self.next_id, self.next_id + 1
        return gid

    def admit(self, gid: int, packet: dict) -> None:
        self.slots[gid] = [packet, False]

    def take(self):
        for slot in self.slots.values():
            if not slot[1]:
                slot[1] = True
                return slot[0]
        return None

    def retire(self, consumed, dropped) -> dict:
        ids = sorted([*consumed, *dropped])
        oldest = list(self.slots)[:len(ids)]
        if len(set(ids)) != len(ids) or ids != oldest or not all(self.slots[g][1] for g in ids):
            raise ValueError("commit requires the delivered oldest group prefix without duplicates")
        for gid in ids:
            del self.slots[gid]
        if ids:
            self.highwater = ids[-1] + 1
        self.dropped += len(dropped)
        return {"committed_highwater": self.highwater, "dropped_groups": self.dropped}

    def pending(self) -> list:
        return [_pack(packet) for packet, _ in self.slots.values()]


class _Sampler:
    """The child's policy, RNG and reward; ``sample(group_id)`` produces one group packet."""

    def __init__(self, settings: dict) -> None:
        from .checkpoint import load_policy_artifact
        from .data import PromptRecord, build_reward
        from .rollout import generation_options
        from .runtime import make_model
        from .tokenizer import ModelTokenizer

        config = self.config = settings["config"]
        torch.set_num_threads(config.num_threads)
        self.records = [PromptRecord(**fields) for fields in settings["records"]]
        model_dir = settings["model_dir"]
        self.model = make_model(model_dir, settings["model_config"], config, config.rollout_devices,
                                settings["random_init"], role="rollout")
        self.model.eval()  # sampling runs under inference_mode; the trainable partition matches the learner's
        has_tokenizer = (Path(model_dir) / "tokenizer.json").is_file()
        self.reward_fn = build_reward(config.reward, tokenizer=ModelTokenizer(model_dir) if has_tokenizer else None)
        self.generation = generation_options(model_dir, settings["model_config"], config)
        self.generator = torch.Generator(device="cpu")
        if settings["rng_state"] is None:
            self.generator.manual_seed(config.seed)
        else:
            self.generator.set_state(settings["rng_state"])
        self._load = load_policy_artifact
        self.receipt: dict = {}
        self.artifact: dict = {}
        self.activate(settings["initial_policy"])

    def activate(self, artifact: dict) -> dict:
        self.receipt = dict(self._load(self.model, artifact))
        self.artifact = dict(artifact)
        return dict(self.receipt)

    def sample(self, group_id: int) -> dict:
        from .rollout import generate_group

        cfg = self.config
        started = time.monotonic()
        group = generate_group(self.model, self.records[group_id % len(self.records)], cfg.group_size,
                               cfg.max_new_tokens, cfg.temperature, policy_version=self.receipt["version"],
                               group_id=group_id, generator=self.generator, reward_fn=self.reward_fn,
                               **self.generation)
        return {"group": group, "policy_ack": dict(self.receipt), "started_at": started,
                "finished_at": time.monotonic(), "engram_shared": False}

    def evaluate(self, records, *, step, phase) -> dict:
        from .data import PromptRecord
        from .evaluation import evaluate_policy

        metrics, rows = evaluate_policy(self.model, [PromptRecord(**fields) for fields in records], self.config,
                                        reward_fn=self.reward_fn, generation_kwargs=self.generation, step=step,
                                        phase=phase, return_rows=True)
        return {"metrics": metrics, "rows": rows}


class _ChildLoop:
    """Request handlers of the child; one group is sampled between polls while admission is open."""

    def __init__(self, settings: dict) -> None:
        config = self.config = settings["config"]
        recovery = settings["recovery_state"] or {}
        if recovery:
            lineage = recovery.get("active_policy", {}).get("lineage")
            if recovery.get("schema_version") != SNAPSHOT_SCHEMA or lineage != settings["initial_policy"]["lineage"]:
                raise ValueError("manager recovery schema or policy lineage differs")
            if recovery.get("rng_state") is not None:
                settings = dict(settings, rng_state=recovery["rng_state"])
        self.box = _Mailbox.restore(recovery, config.queue_capacity + config.groups_per_step,
                                    settings["next_group_id"])
        self.sampler = _Sampler(settings)
        self.paused = bool(settings["start_paused"])
        self.resume_epoch = settings["resume_epoch"]
        self.closing = False
        self.handlers = {"get": self.on_get, "pause": self.on_pause, "commit": self.on_commit,
                         "activate": self.on_activate, "evaluate": self.on_evaluate, "resume": self.on_resume,
                         "close": self.on_close}

    def snapshot(self) -> dict:
        box, sampler = self.box, self.sampler
        return {"schema_version": SNAPSHOT_SCHEMA, "next_group_id": box.next_id,
                "committed_highwater": box.highwater, "dropped_groups": box.dropped,
                "rng_state": sampler.generator.get_state().numpy().tobytes(), "pending_packets": box.pending(),
                "active_policy": dict(sampler.artifact), "policy_ack": dict(sampler.receipt),
                "queue_capacity": self.config.queue_capacity, "retained_capacity": box.bound,
                "admission_paused": True, "resume_epoch": self.resume_epoch}

    def on_get(self, request):
        packet = self.box.take()
        return None if packet is None else _pack(packet)

    def on_pause(self, request):
        self.paused = True
        return self.snapshot()

    def on_commit(self, request):
        return self.box.retire(request["consumed"], request["dropped"])

    def on_activate(self, request):
        if not self.paused:
            raise ValueError("activation requires pause() first")
        return self.sampler.activate(request["artifact"])

    def on_evaluate(self, request):
        if not self.paused:
            raise ValueError("evaluation requires a paused manager")
        return self.sampler.evaluate(request["records"], step=request["step"], phase=request["phase"])

    def on_resume(self, request):
        self.paused = False
        return dict(self.sampler.receipt)

    def on_close(self, request):
        self.closing = True
        return {"cleanup": "drained", "recovery": self.snapshot()}

    def run(self, connection) -> None:
        connection.send({"id": 0, "value": dict(self.sampler.receipt)})
        while not self.closing:
            while connection.poll():
                try:
                    request = connection.recv()
                except EOFError:
                    return
                handler = self.handlers.get(request["command"])
                if handler is None:
                    raise ValueError("unknown manager command: " + str(request["command"]))
                connection.send({"id": request["id"], "value": handler(request)})
                if self.closing:
                    return
            if not self.paused and self.box.has_room(self.config.queue_capacity):
                gid = self.box.reserve()  # the cursor moves before sampling
                self.box.admit(gid, self.sampler.sample(gid))
            else:
                time.sleep(0.005)


def _child_main(connection, settings) -> None:
    try:
        _ChildLoop(settings).run(connection)
    except BaseException:
        try:
            connection.send({"fatal": traceback.format_exc()})
        except (EOFError, BrokenPipeError, OSError):
            pass
    finally:
        connection.close()


class _Link:
    """Learner end of the pipe: numbered requests, deadline-bounded replies, sticky failure."""

    def __init__(self, connection, process, timeout: float) -> None:
        self.connection = connection
        self.process = process
        self.timeout = timeout
        self.counter = 0
        self.failed = False

    def _fail(self, message: str):
        self.failed = True
        return RuntimeError("rollout worker failed: " + message)

    def reply(self, request_id: int):
        deadline = time.monotonic() + self.timeout
        while True:
            left = deadline - time.monotonic()
            if left <= 0:
                self.failed = True
                raise TimeoutError("rollout worker failed: manager command acknowledgement timed out")
            if self.connection.poll(min(0.05, left)):
                try:
                    message = self.connection.recv()
                except EOFError:
                    raise self._fail("manager process closed its channel") from None
                if "fatal" in message:
                    raise self._fail("\n" + message["fatal"])
                if message["id"] != request_id:
                    raise self._fail("manager reply identity differs")
                return message["value"]
            if not self.process.is_alive():
                raise self._fail(f"manager process exited with code {self.process.exitcode}")

    def call(self, command: str, **fields):
        self.counter += 1
        try:
            self.connection.send({"id": self.counter, "command": command, **fields})
        except (BrokenPipeError, EOFError, OSError):
            if not self.connection.poll():  # a fatal report may already be waiting
                raise self._fail("manager command channel closed") from None
        return self.reply(self.counter)


class RolloutManager:
    """Learner-side handle of the rollout child (see the module docstring for the contract)."""

    def __init__(self, model_dir, model_config, config, records, random_init=False, *, initial_policy,
                 recovery_state=None, next_group_id=0, rng_state=None, event_root=None, start_paused=False,
                 engram_weights=None) -> None:
        if not records:
            raise ValueError("manager requires at least one prompt record")
        self.config = config
        self.settings = {"model_dir": str(Path(model_dir).resolve()), "model_config": model_config, "config": config,
                         "records": [asdict(r) for r in records], "random_init": random_init,
                         "initial_policy": dict(initial_policy), "recovery_state": recovery_state,
                         "next_group_id": next_group_id, "rng_state": rng_state,
                         "event_root": None if event_root is None else str(event_root),
                         "resume_epoch": uuid.uuid4().hex, "start_paused": bool(start_paused)}
        self.process = None
        self._link: _Link | None = None
        self._closed = False

    @property
    def pid(self):
        return None if self.process is None else self.process.pid

    def start(self):
        if self.process is not None or self._closed:
            raise ValueError("manager start is single-use")
        context = mp.get_context("spawn")
        parent, child = context.Pipe()
        self.process = context.Process(target=_child_main, args=(child, self.settings), name="tdsv-rollout-manager")
        self.process.start()
        child.close()
        self._link = _Link(parent, self.process, self.config.worker_timeout_seconds)
        return self._link.reply(0)

    def _call(self, command: str, **fields):
        if self._link is None or self._closed or self._link.failed:
            raise RuntimeError("manager is not running")
        return self._link.call(command, **fields)

    def get(self, timeout=None) -> dict:
        deadline = time.monotonic() + (self.config.worker_timeout_seconds if timeout is None else timeout)
        while True:
            packet = self._call("get")
            if packet is not None:
                return _unpack(packet)
            left = deadline - time.monotonic()
            if left <= 0:
                raise queue.Empty
            time.sleep(min(0.01, left))

    def pause(self):
        return _rng_as_tensor(self._call("pause"))

    def commit(self, consumed_group_ids=(), dropped_group_ids=()):
        return self._call("commit", consumed=list(consumed_group_ids), dropped=list(dropped_group_ids))

    def activate(self, artifact):
        return self._call("activate", artifact=dict(artifact))

    def resume(self):
        return self._call("resume")

    def evaluate(self, records, *, step, phase="eval"):
        return self._call("evaluate", records=[asdict(r) for r in records], step=step, phase=phase)

    def close(self):
        """Drain and stop the child (idempotent). A failure seen here is raised unless an earlier
        call already reported the child as failed."""
        if self._closed:
            return None
        link = self._link
        failed_before = link is not None and link.failed
        error, result = None, None
        try:
            if link is not None and self.process.is_alive() and not failed_before:
                result = link.call("close")
        except (RuntimeError, TimeoutError, BrokenPipeError, EOFError, OSError) as exc:
            error = exc
        finally:
            self._closed = True
            if self.process is not None:
                if not _reap(self.process):
                    error = error or RuntimeError("manager cleanup failed to drain its sampler")
                if link is not None:
                    link.connection.close()
        if error is not None and not failed_before:
            raise error
        if result is not None:
            result = dict(result, recovery=_rng_as_tensor(result.get("recovery")))
        return result


def _reap(process) -> bool:
    """Join the owned child; escalate to terminate / kill when it does not exit. True if it exited."""
    process.join(timeout=5)
    if not process.is_alive():
        return True
    process.terminate()
    process.join(timeout=5)
    if process.is_alive():
        process.kill()
        process.join()
    return False


def _rng_as_tensor(snapshot):
    """The child sends its generator state as bytes (a tensor would cross the pipe as a shared-memory
    descriptor that the child's exit can revoke before the learner reads it); callers and
    checkpoints get a uint8 tensor."""
    if snapshot and isinstance(snapshot.get("rng_state"), (bytes, bytearray)):
        snapshot = dict(snapshot, rng_state=torch.frombuffer(bytearray(snapshot["rng_state"]), dtype=torch.uint8))
    return snapshot


__all__ = ["RolloutManager", "SNAPSHOT_SCHEMA"]
