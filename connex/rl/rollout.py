"""Rollout pool: route rollouts over elastic engine instances so that no
request ever mixes two weight versions.

Invariant: a request is bound to the pool's version when admitted and runs
only on an instance at exactly that version, and an instance changes
version only while no request is in flight on it.  Hence:

* ``add``: a new instance first catches up to the pool's version;
* ``update(v, rolling=k)``: the pool moves to ``v`` at once (new requests
  wait for an instance at ``v``), then updates ``k`` instances at a time --
  each stops admitting, drains (or, past ``drain_timeout``, has its
  requests aborted; they restart at ``v``), updates and serves again;
* an instance that dies mid-request is dropped; the request continues on
  another instance of the same version (from the tokens so far when the
  instance ``supports_resume``), or restarts at the pool's version when
  that version is gone; an instance that fails its update is dropped.

Each request is a small state machine (:class:`_Rollout`): bound version,
tokens produced so far, instances tried, attempts.
Behavioural parity: ``connex/rl/rollout.py:32-237`` of the reference.
"""
from __future__ import annotations

import asyncio
import enum
import logging
import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional

log = logging.getLogger("connex.rl.rollout")


class InstanceState(enum.Enum):
    JOINING = "joining"
    SERVING = "serving"
    UPDATING = "updating"
    DEAD = "dead"


class InstanceDead(Exception):
    """The instance's engine died; ``partial`` holds the tokens generated so far."""

    def __init__(self, msg: str = "", partial=None):
        super().__init__(msg)
        self.partial = list(partial or [])


class Aborted(Exception):
    """The pool aborted the request on this instance (for an update)."""


class RolloutInstance:
    """What the pool drives (``FakeInstance`` in tests, HTTP engines in
    :mod:`connex.rl.engines`)."""

    name = "instance"
    version = None
    supports_resume = False

    async def generate(self, req, partial=None):
        raise NotImplementedError

    async def abort_all(self):
        pass

    async def update(self, version):
        raise NotImplementedError

    async def close(self):
        pass


class _Seat:
    """The pool's view of one instance: its state and its requests in flight."""

    def __init__(self, inst: RolloutInstance):
        self.inst = inst
        self.state = InstanceState.JOINING
        self.running: set = set()
        self.quiet = asyncio.Event()
        self.quiet.set()

    @property
    def load(self) -> int:
        return len(self.running)

    def admit(self, key) -> None:
        self.running.add(key)
        self.quiet.clear()

    def finish(self, key) -> None:
        self.running.discard(key)
        if not self.running:
            self.quiet.set()


@dataclass
class _Rollout:
    version: int
    tokens: List[int] = field(default_factory=list)      # produced before a death, for resume
    tried: List[str] = field(default_factory=list)
    attempts: int = 0

    def rebind(self, version: int) -> None:
        """Start over at ``version`` (nothing carried over)."""
        self.version, self.tokens, self.tried = version, [], []


class RolloutPool:
    def __init__(self, version: int = 0, drain_timeout: Optional[float] = None, max_attempts: int = 6):
        self.version = version
        self.drain_timeout = drain_timeout
        self.max_attempts = max_attempts
        self.slots: Dict[str, _Seat] = {}
        self.changed = asyncio.Condition()
        self.stats = {"requests": 0, "completed": 0, "restarted": 0, "resumed": 0, "aborted_for_update": 0,
                      "instance_failures": 0, "failed": 0, "tokens": 0, "updates": []}

    async def _wake(self) -> None:
        async with self.changed:
            self.changed.notify_all()

    async def _move(self, seat: _Seat, state: InstanceState) -> None:
        seat.state = state
        await self._wake()

    # ------------------------------------------------------------ instances
    async def add(self, inst: RolloutInstance) -> None:
        seat = self.slots[inst.name] = _Seat(inst)
        if inst.version != self.version:
            try:
                await inst.update(self.version)
            except Exception as e:
                log.warning("%s could not catch up to v%s: %s", inst.name, self.version, e)
                self.slots.pop(inst.name, None)
                raise
        # an instance that came up ahead of the pool waits until the pool moves there
        await self._move(seat, InstanceState.SERVING if inst.version == self.version else InstanceState.JOINING)

    async def remove(self, name: str, drain: bool = True) -> None:
        seat = self.slots.get(name)
        if seat is None:
            return
        await self._move(seat, InstanceState.UPDATING)
        if drain:
            await seat.quiet.wait()
        else:
            await self._abort(seat)
        self.slots.pop(name, None)
        await seat.inst.close()
        await self._wake()

    def mark_dead(self, name: str) -> None:
        seat = self.slots.pop(name, None)
        if seat is not None:
            seat.state = InstanceState.DEAD
            self.stats["instance_failures"] += 1

    def serving(self, version=None) -> List[_Seat]:
        want = self.version if version is None else version
        return [s for s in self.slots.values() if s.state is InstanceState.SERVING and s.inst.version == want]

    # -------------------------------------------------------------- requests
    async def _seat_for(self, ro: _Rollout) -> Optional[_Seat]:
        """The least loaded instance serving ``ro.version`` (one not tried yet
        if possible); waits for one; None when that version is gone."""
        async with self.changed:
            while True:
                ready = self.serving(ro.version)
                fresh = [s for s in ready if s.inst.name not in ro.tried] or ready
                if fresh:
                    return min(fresh, key=lambda s: s.load)
                if ro.version != self.version:
                    return None
                await self.changed.wait()

    async def _attempt(self, seat: _Seat, req, ro: _Rollout) -> List[int]:
        resume = ro.tokens if ro.tokens and seat.inst.supports_resume else None
        if resume is None:
            ro.tokens = []
        out = await seat.inst.generate(req, partial=resume)
        return list(resume or []) + list(out["tokens"])

    async def generate(self, req) -> dict:
        """One rollout -> ``{"tokens", "version", "instance", "attempts"}``."""
        self.stats["requests"] += 1
        ro = _Rollout(self.version)
        key = object()
        while ro.attempts < self.max_attempts:
            seat = await self._seat_for(ro)
            if seat is None:                       # its version is gone: restart at the pool's
                ro.rebind(self.version)
                self.stats["restarted"] += 1
                continue
            ro.attempts += 1
            seat.admit(key)
            try:
                tokens = await self._attempt(seat, req, ro)
                self.stats["completed"] += 1
                self.stats["tokens"] += len(tokens)
                return {"tokens": tokens, "version": ro.version, "instance": seat.inst.name, "attempts": ro.attempts}
            except Aborted:
                self.stats["aborted_for_update"] += 1
                ro.rebind(self.version)
            except InstanceDead as e:
                log.warning("instance %s died during a request", seat.inst.name)
                self.mark_dead(seat.inst.name)
                ro.tried.append(seat.inst.name)
                if seat.inst.supports_resume and e.partial:
                    ro.tokens = list(ro.tokens) + e.partial
                    self.stats["resumed"] += 1
            finally:
                seat.finish(key)
        self.stats["failed"] += 1
        raise RuntimeError(f"request failed after {ro.attempts} attempts")

    # --------------------------------------------------------------- updates
    async def _abort(self, seat: _Seat) -> None:
        if seat.running:
            await seat.inst.abort_all()
            await seat.quiet.wait()

    async def _quiesce(self, seat: _Seat) -> None:
        """No request in flight on ``seat`` any more (drained, or aborted after the timeout)."""
        if self.drain_timeout is None:
            await seat.quiet.wait()
            return
        try:
            await asyncio.wait_for(seat.quiet.wait(), self.drain_timeout)
        except asyncio.TimeoutError:
            await self._abort(seat)

    async def _update_one(self, seat: _Seat, version) -> bool:
        await self._move(seat, InstanceState.UPDATING)
        await self._quiesce(seat)
        try:
            if seat.inst.version != version:
                await seat.inst.update(version)
            if seat.inst.version != version:
                raise RuntimeError(f"came up at v{seat.inst.version}, wanted v{version}")
        except Exception as e:  # noqa: BLE001 - the instance is dropped
            log.warning("%s failed to update to v%s: %s; removing it", seat.inst.name, version, e)
            self.mark_dead(seat.inst.name)
            await self._wake()
            return False
        await self._move(seat, InstanceState.SERVING)
        return True

    async def update(self, version, rolling: Optional[int] = None) -> int:
        """Move the pool to ``version``; returns how many instances updated."""
        t0 = time.perf_counter()
        self.version = version
        await self._wake()
        seats = list(self.slots.values())
        width = rolling or len(seats) or 1
        updated = 0
        for start in range(0, len(seats), width):
            wave = seats[start:start + width]
            updated += sum(await asyncio.gather(*(self._update_one(s, version) for s in wave)))
        self.stats["updates"].append({"version": version, "s": time.perf_counter() - t0, "instances": updated,
                                      "of": len(seats)})
        return updated
