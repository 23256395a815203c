"""Fake rollout engine for CPU tests and churn simulations (reference
``connex/rl/fake.py:19-77``).

Its model is one scalar pulled through a real :class:`WeightSubscriber`;
token ``i`` of a request is a pure function of ``(seed, i, weight)``, so a
test can tell whether every token of a response came from one version.
"""
from __future__ import annotations

import asyncio

import torch

from .rollout import Aborted, InstanceDead, RolloutInstance


def token(seed: int, i: int, w) -> int:
    return int((seed * 1000003 + i * 7919 + int(w)) % 50000)


def expected(req, w):
    return [token(req["seed"], i, w) for i in range(req["max_tokens"])]


def weights_for(version: int, n: int = 4096):
    return [("w", torch.full((n,), float(version))), ("b", torch.arange(16.0) + version)]


class FakeInstance(RolloutInstance):
    supports_resume = True

    def __init__(self, name: str, subscriber=None, tpot_s: float = 0.001, update_s: float = 0.0):
        self.name = name
        self.sub = subscriber
        self.version = None
        self.w = None
        self.tpot_s = tpot_s
        self.update_s = update_s
        self.dead = False
        self._abort = asyncio.Event()
        self.served = 0

    def kill(self) -> None:
        self.dead = True

    async def generate(self, req, partial=None):
        if self.dead:
            raise InstanceDead("down")
        w, out = self.w, []
        for i in range(len(partial or []), req["max_tokens"]):
            await asyncio.sleep(self.tpot_s)
            if self.dead:
                raise InstanceDead("died", partial=out)
            if self._abort.is_set():
                raise Aborted()
            out.append(token(req["seed"], i, w))
        self.served += 1
        return {"tokens": out}

    async def abort_all(self):
        self._abort.set()
        await asyncio.sleep(self.tpot_s * 2)
        self._abort.clear()

    async def update(self, version):
        if self.dead:
            raise InstanceDead("down")
        await asyncio.sleep(self.update_s)
        if self.sub is None:
            self.w, self.version = float(version), version
            return

        def apply(named):
            for _, t in named:
                self.w = float(t.view(-1)[0])
                break
        st = await asyncio.to_thread(self.sub.sync, apply, version)
        self.version = st["version"]
