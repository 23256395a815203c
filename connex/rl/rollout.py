"""Rollout pool: route rollouts over elastic engine instances so that no
request ever mixes two weight versions (reference ``connex/rl/rollout.py:63-237``).

A request takes the pool's version when admitted and runs only on an
instance at exactly that version.  Instances change version only with no
request in flight (drained, or aborted and re-queued), so:

* ``add``: the instance catches up to the pool version before serving;
* ``update(v, rolling=k)``: new requests wait for an instance at ``v``;
  ``k`` instances at a time stop admitting, drain (or abort past
  ``drain_timeout``; aborted requests restart at ``v``) and update;
* an instance that dies mid-request: the request re-runs on another
  instance of the same version (resuming from the tokens so far when the
  instance ``supports_resume``), else restarts at the pool version; an
  instance that fails its update is removed.
"""
from __future__ import annotations

import asyncio
import enum
import logging
import time
from typing import Dict, List, Optional

log = logging.getLogger("connex.rl.rollout")


class InstanceState(enum.Enum):
    JOINING = "joining"
    SERVING = "serving"
    UPDATING = "updating"
    DEAD = "dead"


class InstanceDead(Exception):
    """The instance's engine died; ``partial`` = tokens generated so far."""

    def __init__(self, msg: str = "", partial=None):
        super().__init__(msg)
        self.partial = list(partial or [])


class Aborted(Exception):
    """The pool aborted the request on this instance (for an update)."""


class RolloutInstance:
    """What the pool drives (``FakeInstance`` for tests, HTTP engines in
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


class _Member:
    def __init__(self, inst: RolloutInstance):
        self.inst = inst
        self.state = InstanceState.JOINING
        self.inflight: Dict = {}
        self.idle = asyncio.Event()
        self.idle.set()

    def enter(self, task, req) -> None:
        self.inflight[task] = req
        self.idle.clear()

    def leave(self, task) -> None:
        self.inflight.pop(task, None)
        if not self.inflight:
            self.idle.set()


class RolloutPool:
    def __init__(self, version: int = 0, drain_timeout: Optional[float] = None, max_attempts: int = 6):
        self.version = version
        self.drain_timeout = drain_timeout
        self.max_attempts = max_attempts
        self.slots: Dict[str, _Member] = {}
        self.changed = asyncio.Condition()
        self.stats = {"requests": 0, "completed": 0, "restarted": 0, "resumed": 0, "aborted_for_update": 0,
                      "instance_failures": 0, "failed": 0, "tokens": 0, "updates": []}

    async def _notify(self) -> None:
        async with self.changed:
            self.changed.notify_all()

    async def _set(self, m: _Member, state: InstanceState) -> None:
        m.state = state
        await self._notify()

    # ---------------------------------------------------------- membership
    async def add(self, inst: RolloutInstance) -> None:
        m = _Member(inst)
        self.slots[inst.name] = m
        if inst.version != self.version:
            try:
                await inst.update(self.version)
            except Exception as e:
                log.warning("%s could not catch up to v%s: %s", inst.name, self.version, e)
                self.slots.pop(inst.name, None)
                raise
        # came up ahead of the pool (next version already published): park it
        await self._set(m, InstanceState.SERVING if inst.version == self.version else InstanceState.JOINING)

    async def remove(self, name: str, drain: bool = True) -> None:
        m = self.slots.get(name)
        if m is None:
            return
        await self._set(m, InstanceState.UPDATING)
        if drain:
            await m.idle.wait()
        else:
            await self._abort(m)
        self.slots.pop(name, None)
        await m.inst.close()
        await self._notify()

    def mark_dead(self, name: str) -> None:
        m = self.slots.pop(name, None)
        if m is not None:
            m.state = InstanceState.DEAD
            self.stats["instance_failures"] += 1

    def serving(self, version=None) -> List[_Member]:
        v = self.version if version is None else version
        return [m for m in self.slots.values() if m.state is InstanceState.SERVING and m.inst.version == v]

    # ------------------------------------------------------------ requests
    async def _pick(self, version, exclude=()):
        async with self.changed:
            while True:
                ok = self.serving(version)
                pref = [m for m in ok if m.inst.name not in exclude] or ok
                if pref:
                    return min(pref, key=lambda m: len(m.inflight))
                if version != self.version:
                    return None          # the old version is gone
                await self.changed.wait()

    async def generate(self, req) -> dict:
        """One rollout -> ``{"tokens", "version", "instance", "attempts"}``."""
        self.stats["requests"] += 1
        version, partial, tried, attempts = self.version, [], [], 0
        task = asyncio.current_task()
        while attempts < self.max_attempts:
            m = await self._pick(version, tried)
            if m is None:
                version, partial, tried = self.version, [], []
                self.stats["restarted"] += 1
                continue
            attempts += 1
            m.enter(task, req)
            try:
                resume = partial if (partial and m.inst.supports_resume) else None
                if partial and resume is None:
                    partial = []
                out = await m.inst.generate(req, partial=resume)
                toks = list(resume or []) + list(out["tokens"])
                self.stats["completed"] += 1
                self.stats["tokens"] += len(toks)
                return {"tokens": toks, "version": version, "instance": m.inst.name, "attempts": attempts}
            except Aborted:
                self.stats["aborted_for_update"] += 1
                version, partial, tried = self.version, [], []
            except InstanceDead as e:
                log.warning("instance %s died during a request", m.inst.name)
                self.mark_dead(m.inst.name)
                tried.append(m.inst.name)
                if m.inst.supports_resume and e.partial:
                    partial = list(partial) + e.partial
                    self.stats["resumed"] += 1
            finally:
                m.leave(task)
        self.stats["failed"] += 1
        raise RuntimeError(f"request failed after {attempts} attempts")

    # ------------------------------------------------------------- updates
    async def _abort(self, m: _Member) -> None:
        if m.inflight:
            await m.inst.abort_all()
            await m.idle.wait()

    async def _update_one(self, m: _Member, version) -> bool:
        await self._set(m, InstanceState.UPDATING)
        if self.drain_timeout is None:
            await m.idle.wait()
        else:
            try:
                await asyncio.wait_for(m.idle.wait(), self.drain_timeout)
            except asyncio.TimeoutError:
                await self._abort(m)
        try:
            if m.inst.version != version:
                await m.inst.update(version)
            if m.inst.version != version:
                raise RuntimeError(f"came up at v{m.inst.version}, wanted v{version}")
        except Exception as e:  # noqa: BLE001
            log.warning("%s failed to update to v%s: %s; removing it", m.inst.name, version, e)
            self.mark_dead(m.inst.name)
            await self._notify()
            return False
        await self._set(m, InstanceState.SERVING)
        return True

    async def update(self, version, rolling: Optional[int] = None) -> int:
        """Move the pool to ``version``; returns how many instances updated."""
        t0 = time.perf_counter()
        self.version = version
        await self._notify()
        members = list(self.slots.values())
        k = rolling or len(members) or 1
        ok = 0
        for i in range(0, len(members), k):
            ok += sum(await asyncio.gather(*(self._update_one(m, version) for m in members[i:i + k])))
        self.stats["updates"].append({"version": version, "s": time.perf_counter() - t0, "instances": ok,
                                      "of": len(members)})
        return ok
