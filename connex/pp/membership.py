"""Pipeline membership from the directory (reference ``connex/directory.py``
clients as used by stage endpoints).

:class:`DirectoryMembership` gives a :class:`connex.pp.endpoint.PipelineEndpoint`
the membership surface it routes with -- ``get_pipeline_peers()``,
``get_stage_peers(stage)``, ``on_event(EventType, callback)`` -- from a
:class:`connex.directory.DirectoryClient`: routes come from ``list_stage``
(cached; refreshed on every membership event) and directory ``LEAVE`` events
(deregister or lease expiry) are delivered as ``ENDPOINT_DEREGISTERED``.
"""
from __future__ import annotations

import threading
from collections import defaultdict
from typing import Callable, Dict, List

from connex.front_router import EventType
from connex.pp.routing import Lid, Route


class _Event:
    def __init__(self, payload: dict):
        self.payload = payload


class DirectoryMembership:
    def __init__(self, client, num_stages: int):
        self.client = client
        self.num_stages = num_stages
        self._routes: Dict[int, List[Route]] = {}
        self._lock = threading.Lock()
        self._handlers: Dict[int, list] = defaultdict(list)
        client.subscribe_events(self._on_directory_event)

    def refresh_routes(self) -> None:
        with self._lock:
            self._routes.clear()

    def get_stage_peers(self, stage_idx: int, refresh: str = "auto") -> List[Route]:
        with self._lock:
            hit = self._routes.get(stage_idx)
        if hit is None or refresh == "always":
            infos = self.client.list_stage(stage_idx) or []
            hit = [Route(Lid(i.lid[1], i.lid[3], i.lid[0]), list(i.addresses)) for i in infos]
            with self._lock:
                self._routes[stage_idx] = hit
        return list(hit)

    def get_pipeline_peers(self) -> List[Route]:
        out: List[Route] = []
        for s in range(self.num_stages):
            out += self.get_stage_peers(s)
        return out

    def on_event(self, event_type, callback: Callable) -> None:
        self._handlers[int(event_type)].append(callback)

    def _on_directory_event(self, event, info) -> None:
        self.refresh_routes()
        kind = getattr(event, "value", event)
        et = {"LEAVE": EventType.ENDPOINT_DEREGISTERED, "JOIN": EventType.ENDPOINT_REGISTERED,
              "MIGRATE": EventType.ENDPOINT_REGISTERED}.get(kind)
        if et is None:
            return
        ev = _Event({"lid": {"model_name": info.lid[0], "stage_idx": info.lid[1], "shard_idx": info.lid[2],
                             "replica_idx": info.lid[3]}, "reason": "left" if kind == "LEAVE" else "",
                     "addresses": list(info.addresses)})
        for cb in list(self._handlers.get(int(et), ())):
            cb(ev)
