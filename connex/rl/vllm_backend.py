"""``connex`` backend for vLLM's pluggable weight transfer
(``vllm.distributed.weight_transfer``; reference ``connex/rl/vllm_backend.py:57-225``).

Worker side (:class:`ConnexWeightTransferEngine`): ``init_transfer_engine``
joins the weight registry as ``<member>/r<rank>`` with a receive arena;
``receive_weights({"version": v}, load_weights)`` pulls ``v`` from the
trainer or any engine that already holds it (tree fan-out, source failover),
hands the tensors to ``load_weights`` and offers the copy onward.

Trainer side: :meth:`ConnexWeightTransferEngine.trainer_send_weights` packs
the iterator into the publisher's double-buffered arena and publishes the
next version (``trainer_args``: ``{"publisher": WeightPublisher}``, or
``{"registry_url", "transport", "device"}`` to make one).  :class:`PoolClient`
drives many engine clients at once and drops the failed ones.

vLLM is imported only when this module is; :func:`register` adds the backend
to vLLM's factory (``connex.rl.vllm_plugin`` runs it as a general plugin).
"""
from __future__ import annotations

import os
import socket
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass
from typing import Any, Dict, Optional

import torch
from vllm.distributed.weight_transfer.base import (WeightTransferEngine, WeightTransferInitInfo,
                                                   WeightTransferUpdateInfo)

from .registry import RegistryClient
from .sync import DEFAULT_CHUNK, WeightPublisher, WeightSubscriber
from .transport import make_transport

BACKEND = "connex"


@dataclass
class ConnexWeightTransferInitInfo(WeightTransferInitInfo):
    registry_url: str = ""
    member: Optional[str] = None
    transport: str = "engine"          # "engine" | "nvlink" | "local"
    chunk_bytes: int = DEFAULT_CHUNK


@dataclass
class ConnexWeightTransferUpdateInfo(WeightTransferUpdateInfo):
    version: Optional[int] = None      # None: latest


def _make(kind: str, member: str, rank: int):
    if kind in ("local", "nvlink"):
        return make_transport(kind, name=member.replace("/", "-"))
    return make_transport("engine", lid=("connex-rl", 1, rank, os.getpid()))


class ConnexWeightTransferEngine(WeightTransferEngine[ConnexWeightTransferInitInfo,
                                                      ConnexWeightTransferUpdateInfo]):
    init_info_cls = ConnexWeightTransferInitInfo
    update_info_cls = ConnexWeightTransferUpdateInfo

    def __init__(self, config, parallel_config, model):
        super().__init__(config, parallel_config, model)
        self.sub: Optional[WeightSubscriber] = None
        self.transport = None
        self.last_stats: dict = {}

    def _device(self):
        try:
            return next(self.model.parameters()).device
        except (StopIteration, AttributeError):
            return torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else "cpu"

    def init_transfer_engine(self, init_info):
        rank = getattr(self.parallel_config, "rank", 0)
        member = f"{init_info.member or f'{socket.gethostname()}-{os.getpid()}'}/r{rank}"
        if self.transport is None:
            self.transport = _make(init_info.transport, member, rank)
        arena = "host" if init_info.transport == "engine" else "device"
        self.sub = WeightSubscriber(RegistryClient(init_info.registry_url), self.transport, member,
                                    device=self._device(), chunk_bytes=init_info.chunk_bytes, arena=arena)

    def receive_weights(self, update_info, load_weights):
        if self.sub is None:
            raise RuntimeError("connex weight transfer not initialised")
        m = self.sub.pull(update_info.version)
        load_weights(list(self.sub.tensors()))
        dev = torch.device(self._device())
        if dev.type == "cuda":
            torch.cuda.current_stream(dev).synchronize()
        self.sub.commit(m.version)
        self.last_stats = dict(self.sub.stats)

    def shutdown(self):
        if self.sub is not None:
            self.sub.close()
            self.sub = None
        if self.transport is not None:
            self.transport.close()
            self.transport = None

    @staticmethod
    def trainer_send_weights(iterator, trainer_args) -> int:
        pub = trainer_args.get("publisher")
        if pub is None:
            t = make_transport(trainer_args.get("transport", "engine"), name="trainer",
                               lid=("connex-rl", 0, 0, 0))
            pub = WeightPublisher(RegistryClient(trainer_args["registry_url"]), t,
                                  device=trainer_args.get("device", "cpu"), buffers=trainer_args.get("buffers", 2))
            trainer_args["publisher"] = pub
        return pub.publish(list(iterator), trainer_args.get("version"))


class PoolClient:
    """Many engine clients in parallel; a failing one is dropped, not fatal."""

    def __init__(self, clients: Dict[str, Any], on_failure=None):
        self.clients = dict(clients)
        self.on_failure = on_failure
        self.failed: Dict[str, str] = {}

    def _all(self, fn):
        with ThreadPoolExecutor(max_workers=max(1, len(self.clients))) as ex:
            futs = {n: ex.submit(fn, c) for n, c in self.clients.items()}
        for n, f in futs.items():
            try:
                f.result()
            except Exception as e:  # noqa: BLE001
                self.failed[n] = repr(e)
                self.clients.pop(n, None)
                if self.on_failure:
                    self.on_failure(n, e)
        if not self.clients:
            raise RuntimeError(f"every engine failed: {self.failed}")

    def add(self, name, client):
        self.clients[name] = client

    def init_weight_transfer_engine(self, init_info):
        self._all(lambda c: c.init_weight_transfer_engine(dict(init_info)))

    def start_weight_update(self):
        self._all(lambda c: c.start_weight_update())

    def update_weights(self, update_info):
        self._all(lambda c: c.update_weights(update_info))

    def finish_weight_update(self, weight_version=None):
        self._all(lambda c: c.finish_weight_update(weight_version))


_registered = False


def register() -> None:
    """Add the backend to vLLM's factory (idempotent)."""
    global _registered
    if _registered:
        return
    from vllm.distributed.weight_transfer.factory import WeightTransferEngineFactory
    if BACKEND not in WeightTransferEngineFactory._registry:
        WeightTransferEngineFactory.register_engine(BACKEND, ConnexWeightTransferEngine)
    _registered = True
