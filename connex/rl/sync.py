"""Trainer-side publisher and engine-side subscriber (reference
``connex/rl/sync.py:41-259``).

Publisher: pack version ``v`` into one of ``buffers`` registered arenas (the
slot of the oldest version is reused only after its readers drained, or
after ``idle_timeout``, in which case those readers are told their copy is
stale and read again), then announce ``v`` and its manifest.

Subscriber: ask the registry for a source of the latest version, pull the
arena in ``chunk_bytes`` pieces (``window`` in flight), and on a failed read
report the source, take another one and continue from the first chunk that
did not arrive.  The publisher always holds ``v``, so the pull ends while it
lives.  ``apply`` gets the whole version in one call; ``commit`` then offers
the copy to later pullers (tree fan-out) unless ``relay`` is off.
"""
from __future__ import annotations

import logging
import os
import threading
import time
from typing import Callable, Iterable, List, Optional, Tuple

import torch

from .registry import PUBLISHER
from .transport import TransferError
from .weights import WeightManifest, pack_into, unpack

log = logging.getLogger("connex.rl")

DEFAULT_CHUNK = 64 << 20


def _stream_sync(t: Optional[torch.Tensor]) -> None:
    """Wait for the work queued so far on ``t``'s device's current stream only."""
    if t is not None and t.is_cuda:
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(t.device))
        ev.synchronize()


class WeightPublisher:
    def __init__(self, registry, transport, device="cpu", buffers: int = 2, idle_timeout: float = 30.0):
        self.reg = registry
        self.t = transport
        self.device = torch.device(device)
        self.nbuf = max(1, buffers)
        self.arenas: List[list] = []       # [tensor, version]
        self.manifest: Optional[WeightManifest] = None
        self.version = 0
        self.idle_timeout = idle_timeout

    def _slot(self, need: int) -> int:
        if len(self.arenas) < self.nbuf:
            a = torch.empty(need, dtype=torch.uint8, device=self.device)
            self.t.register(a)
            self.arenas.append([a, None])
            return len(self.arenas) - 1
        slot = min(range(self.nbuf), key=lambda i: self.arenas[i][1])
        a, old = self.arenas[slot]
        if old is not None:
            r = self.reg.wait_idle(version=old, member=PUBLISHER, timeout=self.idle_timeout, retire=True)
            if not (r or {}).get("ok", True):
                log.warning("publisher: v%s still read after %.0fs; overwriting (readers re-read)",
                            old, self.idle_timeout)
        if a.numel() < need:
            self.t.unregister(a)
            a = torch.empty(need, dtype=torch.uint8, device=self.device)
            self.t.register(a)
            self.arenas[slot][0] = a
        return slot

    def publish(self, named: Iterable[Tuple[str, torch.Tensor]], version: Optional[int] = None) -> int:
        named = list(named)
        v = self.version + 1 if version is None else version
        m = WeightManifest.build(v, named)
        slot = self._slot(m.total)
        a = self.arenas[slot][0]
        pack_into(a, m, named)
        _stream_sync(a)
        self.arenas[slot][1] = v
        self.reg.publish(version=v, manifest=m.to_dict(), url=self.t.url, addr=a.data_ptr())
        self.version, self.manifest = v, m
        return v


class WeightSubscriber:
    """One per engine worker; ``member`` is its logical id in the registry.

    ``arena``: ``"device"`` (default) or ``"host"`` (pinned host memory, no
    second device copy; env ``CONNEX_RL_ARENA``).  ``relay=False`` (env
    ``CONNEX_RL_RELAY=0``) frees the copy after apply instead of serving it.
    """

    def __init__(self, registry, transport, member: str, device="cpu", chunk_bytes: int = DEFAULT_CHUNK,
                 max_source_failures: int = 16, heartbeat_s: float = 2.0, window: int = 16,
                 arena: Optional[str] = None, relay: Optional[bool] = None):
        self.reg = registry
        self.t = transport
        self.member = member
        arena = arena or os.environ.get("CONNEX_RL_ARENA", "device")
        if arena not in ("device", "host"):
            raise ValueError(f"arena must be 'device' or 'host', got {arena!r}")
        if relay is None:
            relay = os.environ.get("CONNEX_RL_RELAY", "1").lower() not in ("0", "false", "no")
        self.relay = relay
        self.pin = arena == "host" and torch.cuda.is_available()
        self.device = torch.device("cpu") if arena == "host" else torch.device(device)
        self.chunk = chunk_bytes
        self.window = window
        self.max_fail = max_source_failures
        self.arena: Optional[torch.Tensor] = None
        self.manifest: Optional[WeightManifest] = None
        self.version: Optional[int] = None
        self.stats: dict = {}
        self.reg.join(member=member, url=transport.url)
        self._stop = threading.Event()
        if heartbeat_s:
            threading.Thread(target=self._heartbeat, args=(heartbeat_s,), daemon=True).start()

    def _heartbeat(self, every: float) -> None:
        while not self._stop.wait(every):
            try:
                if not self.reg.heartbeat(member=self.member)["ok"]:
                    self.reg.join(member=self.member, url=self.t.url)
            except Exception:  # noqa: BLE001 - the registry may be restarting
                pass

    def latest(self) -> Optional[int]:
        lt = self.reg.get_latest()
        return None if lt is None else lt["version"]

    def pull(self, version: Optional[int] = None) -> WeightManifest:
        """Fetch the latest version (at least ``version``) into the arena."""
        lt = self.reg.get_latest()
        if lt is None:
            raise RuntimeError("no weight version published yet")
        if version is not None and version > lt["version"]:
            lt = self.reg.get_latest(wait_newer_than=version - 1, timeout=60.0)
            if lt is None or lt["version"] < version:
                raise RuntimeError(f"version {version} not published")
        v, m = lt["version"], WeightManifest.from_dict(lt["manifest"])
        t0 = time.perf_counter()
        if self.arena is not None:
            self.reg.retract(member=self.member)   # stop serving the copy about to be overwritten
        self.manifest = None
        for _ in range(3):
            stale, failures, sources = self._read(v, m)
            if not stale:
                break
            log.warning("%s: a source of v%d overwrote its copy mid-read; reading again", self.member, v)
        else:
            raise RuntimeError(f"v{v}: sources kept changing during the read")
        self.manifest = m
        self.stats = {"version": v, "bytes": m.total, "pull_s": time.perf_counter() - t0,
                      "sources": sources, "source_failures": failures}
        return m

    def _release(self, version: int, source: str) -> bool:
        r = self.reg.release(version=version, source=source, member=self.member)
        return bool((r or {}).get("stale"))

    def _ensure_arena(self, total: int) -> None:
        if self.arena is not None and self.arena.numel() >= total:
            return
        if self.arena is not None:
            self.t.unregister(self.arena)
        self.arena = torch.empty(total, dtype=torch.uint8, device=self.device, pin_memory=self.pin)
        _stream_sync(self.arena)   # the previous user of this memory must be done
        self.t.register(self.arena)

    def _read(self, version: int, m: WeightManifest):
        self._ensure_arena(m.total)
        offs = list(range(0, m.total, self.chunk))
        stale, failures, bad, sources = False, 0, set(), []
        src = None
        i = 0
        try:
            while i < len(offs):
                if src is None:
                    src = self.reg.assign(version=version, member=self.member, exclude=sorted(bad))
                    if src is None:
                        raise RuntimeError(f"no source holds version {version}")
                    sources.append(src["member"])
                ops = [(src["addr"] + o, o, min(self.chunk, m.total - o)) for o in offs[i:]]
                try:
                    self.t.read_window(src["url"], ops, self.arena, self.window)
                    i = len(offs)
                except TransferError as e:
                    i += getattr(e, "done", 0)
                    failures += 1
                    log.warning("%s: read of v%d from %s failed (%s); switching source",
                                self.member, version, src["member"], e)
                    self.reg.report_failure(version=version, source=src["member"], reporter=self.member)
                    stale |= self._release(version, src["member"])
                    if src["member"] != PUBLISHER:
                        bad.add(src["member"])
                    src = None
                    if failures > self.max_fail:
                        raise
        except BaseException:
            if src is not None:
                try:
                    self._release(version, src["member"])
                except Exception:  # noqa: BLE001
                    pass
            raise
        if src is not None:
            stale |= self._release(version, src["member"])
        return stale, failures, sources

    def tensors(self):
        return unpack(self.arena, self.manifest)

    def commit(self, version: int) -> None:
        self.version = version
        if self.relay:
            self.reg.done(version=version, member=self.member, url=self.t.url, addr=self.arena.data_ptr())
            return
        self.reg.done(version=version, member=self.member, url=self.t.url, addr=0, hold=False)
        self.t.unregister(self.arena)
        self.arena = self.manifest = None

    def sync(self, apply: Callable, version: Optional[int] = None) -> dict:
        """pull + ``apply(iterable of (name, tensor))`` + commit; returns stats."""
        m = self.pull(version)
        t0 = time.perf_counter()
        apply(self.tensors())
        _stream_sync(self.arena)
        self.stats["apply_s"] = time.perf_counter() - t0
        self.commit(m.version)
        return self.stats

    def close(self, leave: bool = True) -> None:
        self._stop.set()
        if leave:
            try:
                self.reg.leave(member=self.member)
            except Exception:  # noqa: BLE001
                pass
