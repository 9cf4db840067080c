"""Rollout coordinator: bounded, accounted execution of episode plans over benchmark backends
(the role of ``rollout_manager/coordinator.py:18-593``, reduced to its contract).

* Admission: at most ``max_workers`` episodes run at once and at most ``max_groups`` groups are in
  flight; a plan whose benchmark has no backend is rejected before anything runs.
* Every episode gets its own ``CancellationToken``; ``cancel_all`` cancels cooperatively.
* Quarantine: an episode whose result reports an uncertain model request (``request_uncertain``)
  leaves its worker slot quarantined - the slot is never reused in this run, because the remote
  request may still be executing.
* Events (``admitted``, ``started``, ``finished``, ``quarantined``, ``failed``) and immutable
  results go to an ``EventStore`` when one is given.
* ``run_wave`` executes a finite list of plans; ``execute_group`` one group (plans sharing a
  ``group_id``), returning results in plan order.
* Persistent streams (``open_stream`` / ``execute_stream_group`` / ``pause_stream`` /
  ``resume_stream`` / ``close_stream``, the session API of ``coordinator.py:144-260``): backends are
  started once and stay up between groups; each submitted group carries a strictly increasing
  sequence number (a replayed group is refused without remembering every identity), all groups of
  a stream share one run id, and at most ``max_pending`` episodes are submitted and unfinished at
  once. Admission stops for good (the stream's token is cancelled) after a quarantine, an
  infrastructure failure or a result that needs review; ``pause_stream`` waits for the groups in
  flight, and ``close_stream`` pauses and stops the backends.
"""

from __future__ import annotations

import asyncio
import time

from .contracts import CancellationToken, EpisodePlan, EpisodeResult, request_uncertain


class Coordinator:
    def __init__(self, backends: dict, *, max_workers: int = 1, max_groups: int = 1, event_store=None,
                 drain_timeout: float = 600.0) -> None:
        if max_workers < 1 or max_groups < 1:
            raise ValueError("coordinator needs at least one worker and one group slot")
        self.backends = dict(backends)
        self.max_workers, self.max_groups = max_workers, max_groups
        self.store = event_store
        self.drain_timeout = drain_timeout
        self.quarantined = 0
        self.active = 0
        self._slots = None
        self._groups = None
        self._tokens: set[CancellationToken] = set()
        self._stream: dict | None = None

    def _limits(self):
        if self._slots is None:
            self._slots = asyncio.Condition()
            self._groups = asyncio.Semaphore(self.max_groups)

    async def _acquire(self) -> None:
        async with self._slots:
            while self.active + self.quarantined >= self.max_workers:
                if self.quarantined >= self.max_workers:
                    raise RuntimeError("every worker slot is quarantined")
                await self._slots.wait()
            self.active += 1

    async def _release(self, quarantine: bool) -> None:
        async with self._slots:
            self.active -= 1
            if quarantine:
                self.quarantined += 1
            self._slots.notify_all()

    def _event(self, name, plan=None, **details):
        if self.store is not None:
            self.store.append(name, plan.identity if plan is not None else None, **details)

    @property
    def usable_workers(self) -> int:
        return self.max_workers - self.quarantined

    async def _episode(self, plan: EpisodePlan) -> EpisodeResult:
        backend = self.backends[plan.task.benchmark]
        await self._acquire()
        token = CancellationToken()
        self._tokens.add(token)
        quarantine = False
        started = time.monotonic()
        try:
            self._event("started", plan)
            result = await backend.execute(plan, token)
            if request_uncertain(result.request_state):
                quarantine = True  # the slot stays taken: the remote request may still run
                self._event("quarantined", plan, reason="uncertain model request")
            self._event("finished", plan, execution_state=result.execution_state,
                        score_eligible=result.score_eligible, seconds=time.monotonic() - started)
            if self.store is not None:
                self.store.write_result(result)
            return result
        except BaseException as error:
            self._event("failed", plan, error_type=type(error).__name__, reason=str(error)[:2048])
            raise
        finally:
            self._tokens.discard(token)
            await self._release(quarantine)

    def _check(self, plans) -> None:
        missing = {p.task.benchmark for p in plans} - set(self.backends)
        if missing:
            raise ValueError(f"no backend for benchmarks {sorted(missing)}")
        if self.usable_workers < 1:
            raise RuntimeError("every worker slot is quarantined")

    async def execute_group(self, plans: list[EpisodePlan]) -> list[EpisodeResult]:
        self._check(plans)
        if len({p.identity.group_id for p in plans}) != 1:
            raise ValueError("a group's plans must share one group id")
        self._limits()
        async with self._groups:
            for p in plans:
                self._event("admitted", p)
            return list(await asyncio.gather(*(self._episode(p) for p in plans)))

    async def run_wave(self, plans: list[EpisodePlan]) -> list[EpisodeResult]:
        self._check(plans)
        groups: dict[str, list[EpisodePlan]] = {}
        for p in plans:
            groups.setdefault(p.identity.group_id, []).append(p)
        done = await asyncio.gather(*(self.execute_group(g) for g in groups.values()))
        by_plan = {id(p): r for g, rs in zip(groups.values(), done) for p, r in zip(g, rs)}
        return [by_plan[id(p)] for p in plans]

    def cancel_all(self, reason: str = "cancelled") -> None:
        for token in list(self._tokens):
            token.cancel(reason)
        if self._stream is not None:
            self._stream["token"].cancel(reason)

    # -- persistent streams -------------------------------------------------------------------
    async def open_stream(self, *, max_pending: int = 1, cancellation: CancellationToken | None = None) -> None:
        if self._stream is not None or type(max_pending) is not int or max_pending < 1:
            raise ValueError("one stream per coordinator, with a positive pending capacity")
        self._limits()
        started = []
        self._stream = {"token": cancellation or CancellationToken(), "limit": max_pending, "pending": 0,
                        "sequence": -1, "run_id": None, "paused": False, "closed": False, "tasks": set(),
                        "started": started}
        try:
            for backend in self.backends.values():
                if not any(backend is b for b in started):
                    started.append(backend)
                    if hasattr(backend, "start"):
                        await backend.start()
        except BaseException:
            await self.close_stream()
            raise
        self._event("stream_started", pending_limit=max_pending)

    def _stream_open(self) -> dict:
        st = self._stream
        if st is None or st["closed"] or st["paused"] or st["token"].cancelled():
            raise ValueError("stream admission is unavailable")
        return st

    async def execute_stream_group(self, plans, *, sequence: int) -> list[EpisodeResult]:
        """One complete group; results in plan order. Raises before running anything when the group
        is a replay (sequence not above the last), mixes groups or run ids, or exceeds the credit."""
        st = self._stream_open()
        plans = list(plans)
        if (type(sequence) is not int or sequence <= st["sequence"] or not plans
                or len({p.identity for p in plans}) != len(plans)
                or len({p.identity.group_id for p in plans}) != 1):
            raise ValueError("stream requires a new monotonic sequence and one unique complete group")
        run_id = plans[0].identity.run_id
        if any(p.identity.run_id != run_id for p in plans) or st["run_id"] not in (None, run_id):
            raise ValueError("a stream cannot combine run identities")
        if st["pending"] + len(plans) > st["limit"]:
            raise ValueError("bounded stream input credit exhausted")
        self._check(plans)
        st["sequence"], st["run_id"] = sequence, run_id
        st["pending"] += len(plans)
        task = asyncio.current_task()
        st["tasks"].add(task)
        try:
            async with self._groups:
                for p in plans:
                    self._event("admitted", p, sequence=sequence)
                outcomes = await asyncio.gather(*(self._episode(p) for p in plans), return_exceptions=True)
        finally:
            st["pending"] -= len(plans)
            st["tasks"].discard(task)
        results = []
        for plan, outcome in zip(plans, outcomes):
            if isinstance(outcome, BaseException):
                st["token"].cancel("stream_infrastructure_failure")
                raise outcome
            if request_uncertain(outcome.request_state):
                st["token"].cancel("stream_request_unproven")
            elif outcome.failure_category in {"infrastructure", "infrastructure_error"}:
                st["token"].cancel("stream_infrastructure_failure")
            elif outcome.verification_state == "review_required":
                st["token"].cancel("stream_verifier_review_required")
            results.append(outcome)
        return results

    async def pause_stream(self) -> None:
        """Stop admission and wait until the groups already admitted have finished."""
        st = self._stream
        if st is None:
            return
        st["paused"] = True
        others = [t for t in st["tasks"] if t is not asyncio.current_task()]
        if others:
            await asyncio.gather(*others, return_exceptions=True)
        self._event("stream_paused", quarantined=self.quarantined)

    def resume_stream(self) -> None:
        st = self._stream
        if st is None or st["closed"] or st["token"].cancelled():
            raise RuntimeError("stream is closed or admission is stopped")
        st["paused"] = False
        self._event("stream_resumed")

    async def close_stream(self) -> None:
        st = self._stream
        if st is None or st["closed"]:
            return
        await self.pause_stream()
        st["closed"] = True
        for backend in reversed(st["started"]):
            if hasattr(backend, "close"):
                await backend.close()
        self._event("stream_closed", sequence=st["sequence"])


__all__ = ["Coordinator"]
