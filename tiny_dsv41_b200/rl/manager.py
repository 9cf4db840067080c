"""Rollout manager: a spawned child process that samples GRPO groups with the active policy.

Protocol of ``dsv41_train/rl/manager.py:17-357`` (learner-side API and RPC semantics):

* ``start()`` spawns the child, which builds its own policy on the rollout devices, loads the
  initial policy artifact and answers with the activation receipt ``{version, digest, lineage}``.
* ``get(timeout)`` returns the oldest undelivered group packet or raises ``queue.Empty``.
* ``pause()`` stops admission after the group being sampled and returns a recovery snapshot
  (group cursor, committed high-water mark, sampler RNG state, undelivered packets, active policy).
* ``commit(consumed, dropped)`` retires the delivered oldest groups, in order, without gaps.
* ``activate(artifact)`` (paused only) loads a newly published artifact and returns its receipt.
* ``resume()`` restarts admission; ``close()`` drains and stops the child.

The mailbox holds at most ``queue_capacity + groups_per_step`` groups. Every request carries an
id that the reply must echo; a child failure is returned as its traceback. The child samples
synchronously between request polls, so a pause always lands on a group boundary.
"""

from __future__ import annotations

import multiprocessing as mp
import queue
import time
import traceback
import uuid
from dataclasses import asdict
from pathlib import Path

import torch


def _encode(packet: dict) -> dict:
    return {**packet, "group": asdict(packet["group"])}


def _decode(packet: dict) -> dict:
    from .rollout import RolloutGroup, Sample

    value = dict(packet)
    group = value["group"]
    value["group"] = RolloutGroup([Sample(**s) for s in group["samples"]], group["group_id"], group["policy_version"])
    return value


class _Sampler:
    """The child's policy, RNG and reward; ``sample(group_id)`` produces one packet."""

    def __init__(self, settings: dict) -> None:
        import torch

        from .checkpoint import load_policy_artifact
        from .data import PromptRecord, build_reward
        from .rollout import generation_options
        from .runtime import make_model
        from .tokenizer import ModelTokenizer

        config = settings["config"]
        self.config = config
        torch.set_num_threads(config.num_threads)
        self.records = [PromptRecord(**r) for r in settings["records"]]
        model_dir = settings["model_dir"]
        self.model = make_model(model_dir, settings["model_config"], config, config.rollout_devices,
                                settings["random_init"], role="rollout")
        self.model.eval()  # sampling runs under inference_mode; the trainable partition must match the learner
        tokenizer = ModelTokenizer(model_dir) if (Path(model_dir) / "tokenizer.json").is_file() else None
        self.reward_fn = build_reward(config.reward, tokenizer=tokenizer)
        self.generation = generation_options(model_dir, settings["model_config"], config)
        self.generator = torch.Generator(device="cpu")
        if settings["rng_state"] is not None:
            self.generator.set_state(settings["rng_state"])
        else:
            self.generator.manual_seed(config.seed)
        self._load = load_policy_artifact
        self.ack = None
        self.artifact = None
        self.activate(settings["initial_policy"])

    def activate(self, artifact: dict) -> dict:
        self.ack = self._load(self.model, artifact)
        self.artifact = dict(artifact)
        return dict(self.ack)

    def rng_state(self):
        return self.generator.get_state()

    def sample(self, group_id: int) -> dict:
        from .rollout import generate_group

        record = self.records[group_id % len(self.records)]
        started = time.monotonic()
        group = generate_group(self.model, record, self.config.group_size, self.config.max_new_tokens,
                               self.config.temperature, policy_version=self.ack["version"], group_id=group_id,
                               generator=self.generator, reward_fn=self.reward_fn, **self.generation)
        return {"group": group, "policy_ack": dict(self.ack), "started_at": started, "finished_at": time.monotonic(),
                "engram_shared": False}

    def evaluate(self, records, *, step, phase):
        from .data import PromptRecord
        from .evaluation import evaluate_policy

        records = [PromptRecord(**r) for r in records]
        metrics, rows = evaluate_policy(self.model, records, self.config, reward_fn=self.reward_fn,
                                        generation_kwargs=self.generation, step=step, phase=phase, return_rows=True)
        return {"metrics": metrics, "rows": rows}


def _serve(connection, settings: dict) -> None:
    config, recovery = settings["config"], settings["recovery_state"] or {}
    if recovery and (recovery.get("schema_version") != 1
                     or recovery.get("active_policy", {}).get("lineage") != settings["initial_policy"]["lineage"]):
        raise ValueError("manager recovery schema or policy lineage differs")
    if recovery.get("rng_state") is not None:
        settings = dict(settings, rng_state=recovery["rng_state"])
    bound = config.queue_capacity + config.groups_per_step
    next_group = recovery.get("next_group_id", settings["next_group_id"])
    committed = recovery.get("committed_highwater", next_group)
    dropped = recovery.get("dropped_groups", 0)
    retained: dict[int, dict] = {}
    for encoded in recovery.get("pending_packets", []):
        packet = _decode(encoded)
        gid = packet["group"].group_id
        if gid in retained or not committed <= gid < next_group:
            raise ValueError("invalid or duplicate restored group cursor")
        retained[gid] = {"packet": packet, "delivered": False}
    if len(retained) > bound or sorted(retained) != list(range(committed, next_group)):
        raise ValueError("restored mailbox exceeds capacity or has a cursor gap")
    sampler = _Sampler(settings)
    paused = settings["start_paused"]

    def reply(request_id, value=None):
        connection.send({"id": request_id, "value": value})

    def snapshot():
        return {"schema_version": 1, "next_group_id": next_group, "committed_highwater": committed,
                "dropped_groups": dropped, "rng_state": sampler.rng_state().numpy().tobytes(),
                "pending_packets": [_encode(retained[k]["packet"]) for k in sorted(retained)],
                "active_policy": dict(sampler.artifact), "policy_ack": dict(sampler.ack),
                "queue_capacity": config.queue_capacity, "retained_capacity": bound, "admission_paused": True,
                "resume_epoch": settings["resume_epoch"]}

    reply(0, dict(sampler.ack))
    while True:
        while connection.poll():
            try:
                request = connection.recv()
            except EOFError:
                return
            rid, command = request["id"], request["command"]
            if command == "get":
                row = next((r for _, r in sorted(retained.items()) if not r["delivered"]), None)
                if row is None:
                    reply(rid, None)
                else:
                    row["delivered"] = True
                    reply(rid, _encode(row["packet"]))
            elif command == "pause":
                paused = True
                reply(rid, snapshot())
            elif command == "commit":
                ids = sorted([*request["consumed"], *request["dropped"]])
                if (len(set(ids)) != len(ids) or ids != sorted(retained)[:len(ids)]
                        or any(not retained[g]["delivered"] for g in ids)):
                    raise ValueError("commit requires the delivered oldest group prefix without duplicates")
                for g in ids:
                    del retained[g]
                if ids:
                    committed = ids[-1] + 1
                dropped += len(request["dropped"])
                reply(rid, {"committed_highwater": committed, "dropped_groups": dropped})
            elif command == "activate":
                if not paused:
                    raise ValueError("activation requires pause() first")
                reply(rid, sampler.activate(request["artifact"]))
            elif command == "evaluate":
                if not paused:
                    raise ValueError("evaluation requires a paused manager")
                reply(rid, sampler.evaluate(request["records"], step=request["step"], phase=request["phase"]))
            elif command == "resume":
                paused = False
                reply(rid, dict(sampler.ack))
            elif command == "close":
                reply(rid, {"cleanup": "drained", "recovery": snapshot()})
                return
            else:
                raise ValueError("unknown manager command: " + str(command))
        queued = sum(not r["delivered"] for r in retained.values())
        if not paused and len(retained) < bound and queued < config.queue_capacity:
            gid = next_group
            next_group += 1  # reserve the cursor before sampling
            retained[gid] = {"packet": sampler.sample(gid), "delivered": False}
        else:
            time.sleep(0.005)


def _manager_process(connection, settings) -> None:
    try:
        _serve(connection, settings)
    except BaseException:
        try:
            connection.send({"fatal": traceback.format_exc()})
        except (EOFError, BrokenPipeError, OSError):
            pass
    finally:
        connection.close()


class RolloutManager:
    """Synchronous learner-side API over the child's pipe."""

    def __init__(self, model_dir, model_config, config, records, random_init=False, *, initial_policy,
                 recovery_state=None, next_group_id=0, rng_state=None, event_root=None, start_paused=False,
                 engram_weights=None) -> None:
        self.config = config
        self.settings = {"model_dir": str(Path(model_dir).resolve()), "model_config": model_config, "config": config,
                         "records": [asdict(r) for r in records], "random_init": random_init,
                         "initial_policy": dict(initial_policy), "recovery_state": recovery_state,
                         "next_group_id": next_group_id, "rng_state": rng_state,
                         "event_root": str(event_root) if event_root is not None else None,
                         "resume_epoch": uuid.uuid4().hex, "start_paused": bool(start_paused)}
        if not self.settings["records"]:
            raise ValueError("manager requires at least one prompt record")
        self.process = None
        self._request_id = 0
        self._closed = False
        self._failed = False

    @property
    def pid(self):
        return self.process.pid if self.process else None

    def _receive(self, request_id: int, timeout: float):
        deadline = time.monotonic() + timeout
        while True:
            remaining = deadline - time.monotonic()
            if remaining <= 0:
                self._failed = True
                raise TimeoutError("rollout worker failed: manager command acknowledgement timed out")
            if self.connection.poll(min(0.05, remaining)):
                try:
                    response = self.connection.recv()
                except EOFError:
                    self._failed = True
                    raise RuntimeError("rollout worker failed: manager process closed its channel") from None
                if "fatal" in response:
                    self._failed = True
                    raise RuntimeError("rollout worker failed:\n" + response["fatal"])
                if response["id"] != request_id:
                    self._failed = True
                    raise RuntimeError("rollout worker failed: manager reply identity differs")
                return response["value"]
            if not self.process.is_alive():
                self._failed = True
                raise RuntimeError(f"rollout worker failed: manager process exited with code {self.process.exitcode}")

    def start(self):
        if self.process is not None or self._closed:
            raise ValueError("manager start is single-use")
        context = mp.get_context("spawn")
        self.connection, child = context.Pipe()
        self.process = context.Process(target=_manager_process, args=(child, self.settings),
                                       name="tdsv-rollout-manager")
        self.process.start()
        child.close()
        return self._receive(0, self.config.worker_timeout_seconds)

    def _rpc(self, command: str, **values):
        if self.process is None or self._closed or self._failed:
            raise RuntimeError("manager is not running")
        self._request_id += 1
        try:
            self.connection.send({"id": self._request_id, "command": command, **values})
        except (BrokenPipeError, EOFError, OSError):
            if self.connection.poll():
                return self._receive(self._request_id, self.config.worker_timeout_seconds)
            self._failed = True
            raise RuntimeError("rollout worker failed: manager command channel closed") from None
        return self._receive(self._request_id, self.config.worker_timeout_seconds)

    def get(self, timeout=None) -> dict:
        timeout = self.config.worker_timeout_seconds if timeout is None else timeout
        deadline = time.monotonic() + timeout
        while True:
            encoded = self._rpc("get")
            if encoded is not None:
                return _decode(encoded)
            remaining = deadline - time.monotonic()
            if remaining <= 0:
                raise queue.Empty
            time.sleep(min(0.01, remaining))

    def pause(self):
        return _restore_rng_tensor(self._rpc("pause"))

    def commit(self, consumed_group_ids=(), dropped_group_ids=()):
        return self._rpc("commit", consumed=list(consumed_group_ids), dropped=list(dropped_group_ids))

    def activate(self, artifact):
        return self._rpc("activate", artifact=dict(artifact))

    def resume(self):
        return self._rpc("resume")

    def evaluate(self, records, *, step, phase="eval"):
        return self._rpc("evaluate", records=[asdict(r) for r in records], step=step, phase=phase)

    def close(self):
        if self._closed:
            return None
        prior_failure, failure, result = self._failed, None, None
        try:
            if self.process is not None and self.process.is_alive() and not prior_failure:
                result = self._rpc("close")
        except (RuntimeError, TimeoutError, BrokenPipeError, EOFError, OSError) as error:
            failure = error
        finally:
            self._closed = True
            if self.process is not None:
                self.process.join(timeout=5)
                if self.process.is_alive():  # only this owned child is stopped
                    self.process.terminate()
                    self.process.join(timeout=5)
                    if self.process.is_alive():
                        self.process.kill()
                        self.process.join()
                    failure = failure or RuntimeError("manager cleanup failed to drain its sampler")
                self.connection.close()
        if failure and not prior_failure:
            raise failure
        if result is not None:
            result = dict(result, recovery=_restore_rng_tensor(result.get("recovery")))
        return result


def _restore_rng_tensor(snapshot):
    """The child sends its generator state as bytes: a tensor would cross the pipe as a shared-memory
    file descriptor that the child's exit (right after its ``close`` reply) can revoke before the
    parent has fetched it. Callers and checkpoints get the usual uint8 tensor back."""
    if snapshot and isinstance(snapshot.get("rng_state"), (bytes, bytearray)):
        snapshot = dict(snapshot, rng_state=torch.frombuffer(bytearray(snapshot["rng_state"]), dtype=torch.uint8))
    return snapshot


__all__ = ["RolloutManager"]
