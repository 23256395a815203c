"""Fake rollout engine for CPU tests and churn simulations.

The "model" is one scalar weight pulled through a real
:class:`connex.rl.sync.WeightSubscriber` (or set directly).  Token ``i`` of a
request is a pure function of ``(seed, i, weight)`` (:func:`token`), so a
test can check that every token of a response came from one weight version
(:func:`expected`).  Knobs: per-token latency, update latency, ``kill()``
(the next token raises :class:`InstanceDead` with the tokens so far),
``abort_all()`` (in-flight requests raise :class:`Aborted`).

Behavioural parity: ``connex/rl/fake.py:19-77`` of the reference.
"""
from __future__ import annotations

import asyncio

import torch

from .rollout import Aborted, InstanceDead, RolloutInstance

_VOCAB = 50021


def token(seed: int, i: int, w) -> int:
    """The token a fake engine with weight ``w`` emits at position ``i``."""
    return int(((seed + 1) * 2654435761 + (i + 1) * 40503 + int(w) * 97) % _VOCAB)


def expected(req, w):
    return [token(req["seed"], i, w) for i in range(req["max_tokens"])]


def weights_for(version: int, n: int = 4096):
    """A two-tensor "model" whose values identify ``version``."""
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
        self._aborting = asyncio.Event()
        self.served = 0

    def kill(self) -> None:
        self.dead = True

    def _check(self, produced) -> None:
        if self.dead:
            raise InstanceDead("died", partial=produced)
        if self._aborting.is_set():
            raise Aborted()

    async def generate(self, req, partial=None):
        if self.dead:
            raise InstanceDead("down")
        weight, produced = self.w, []
        for i in range(len(partial or []), req["max_tokens"]):
            await asyncio.sleep(self.tpot_s)
            self._check(produced)
            produced.append(token(req["seed"], i, weight))
        self.served += 1
        return {"tokens": produced}

    async def abort_all(self):
        self._aborting.set()
        await asyncio.sleep(2 * self.tpot_s)      # every running request sees it at its next token
        self._aborting.clear()

    async def update(self, version):
        if self.dead:
            raise InstanceDead("down")
        await asyncio.sleep(self.update_s)
        if self.sub is None:
            self.w, self.version = float(version), version
            return

        def apply(named):
            first = next(iter(named))[1]
            self.w = float(first.view(-1)[0])
        stats = await asyncio.to_thread(self.sub.sync, apply, version)
        self.version = stats["version"]
