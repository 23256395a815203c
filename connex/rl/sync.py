"""Trainer-side publisher and engine-side subscriber of elastic weight sync.

:class:`WeightPublisher`
    Packs version ``v`` into one of ``buffers`` registered arenas and
    announces it with its manifest.  The arena slot of the oldest version is
    reused only after its readers drained -- or after ``idle_timeout``, in
    which case the registry tells those readers their copy is stale and they
    read again.

:class:`WeightSubscriber`
    Asks the registry for a source of the latest version and pulls the arena
    as a :class:`_Download`: fixed-size chunks read through a rolling window;
    when a read fails the source is reported, another one is taken and the
    download resumes at the first chunk that did not arrive.  The publisher
    always holds the version, so a download finishes while it lives.  After
    ``apply`` (the whole version in one call) ``commit`` offers the copy to
    later readers (tree fan-out) unless ``relay`` is off.

Behavioural parity: ``connex/rl/sync.py:29-259`` of the reference.
"""
from __future__ import annotations

import logging
import os
import threading
import time
from dataclasses import dataclass, field
from typing import Callable, Iterable, List, Optional, Set, Tuple

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
        self.arenas: List[list] = []       # [tensor, version held]
        self.manifest: Optional[WeightManifest] = None
        self.version = 0
        self.idle_timeout = idle_timeout

    def _new_arena(self, nbytes: int) -> torch.Tensor:
        a = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
        self.t.register(a)
        return a

    def _retire(self, version: int) -> None:
        """Wait (bounded) until nobody reads ``version`` from us any more."""
        r = self.reg.wait_idle(version=version, member=PUBLISHER, timeout=self.idle_timeout, retire=True)
        if not (r or {}).get("ok", True):
            log.warning("publisher: v%s still read after %.0fs; overwriting (readers re-read)", version,
                        self.idle_timeout)

    def _slot(self, need: int) -> int:
        """An arena slot of at least ``need`` bytes for the next version."""
        if len(self.arenas) < self.nbuf:
            self.arenas.append([self._new_arena(need), None])
            return len(self.arenas) - 1
        slot = min(range(self.nbuf), key=lambda i: self.arenas[i][1])
        arena, held = self.arenas[slot]
        if held is not None:
            self._retire(held)
        if arena.numel() < need:
            self.t.unregister(arena)
            self.arenas[slot][0] = self._new_arena(need)
        return slot

    def publish(self, named: Iterable[Tuple[str, torch.Tensor]], version: Optional[int] = None) -> int:
        named = list(named)
        v = self.version + 1 if version is None else version
        manifest = WeightManifest.build(v, named)
        slot = self._slot(manifest.total)
        arena = self.arenas[slot][0]
        pack_into(arena, manifest, named)
        _stream_sync(arena)
        self.arenas[slot][1] = v
        self.reg.publish(version=v, manifest=manifest.to_dict(), url=self.t.url, addr=arena.data_ptr())
        self.version, self.manifest = v, manifest
        return v


@dataclass
class _Download:
    """One version's arena, fetched chunk by chunk from changing sources."""

    version: int
    total: int
    chunk: int
    next_chunk: int = 0                       # first chunk not yet read
    failures: int = 0
    stale: bool = False                       # some source overwrote its copy while we read it
    excluded: Set[str] = field(default_factory=set)
    sources: List[str] = field(default_factory=list)
    source: Optional[dict] = None             # the current assignment

    @property
    def offsets(self) -> List[int]:
        return list(range(0, self.total, self.chunk))

    @property
    def finished(self) -> bool:
        return self.next_chunk >= len(self.offsets)

    def remaining_ops(self) -> list:
        """(remote address, local offset, bytes) of every chunk still missing."""
        base = self.source["addr"]
        return [(base + o, o, min(self.chunk, self.total - o)) for o in self.offsets[self.next_chunk:]]


class WeightSubscriber:
    """One per engine worker; ``member`` is its logical id in the registry.

    ``arena``: ``"device"`` (default) or ``"host"`` (pinned host memory, no
    second device copy; env ``CONNEX_RL_ARENA``).  ``relay=False`` (env
    ``CONNEX_RL_RELAY=0``) frees the copy after apply instead of serving it."""

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
                    self.reg.join(member=self.member, url=self.t.url)     # expired meanwhile: rejoin
            except Exception:  # noqa: BLE001 - the registry may be restarting
                pass

    def latest(self) -> Optional[int]:
        lt = self.reg.get_latest()
        return None if lt is None else lt["version"]

    def _target(self, version: Optional[int]) -> dict:
        lt = self.reg.get_latest()
        if lt is None:
            raise RuntimeError("no weight version published yet")
        if version is not None and version > lt["version"]:
            lt = self.reg.get_latest(wait_newer_than=version - 1, timeout=60.0)
            if lt is None or lt["version"] < version:
                raise RuntimeError(f"version {version} not published")
        return lt

    def pull(self, version: Optional[int] = None) -> WeightManifest:
        """Fetch the latest version (at least ``version``) into the arena."""
        lt = self._target(version)
        v, manifest = lt["version"], WeightManifest.from_dict(lt["manifest"])
        t0 = time.perf_counter()
        if self.arena is not None:
            self.reg.retract(member=self.member)     # stop serving the copy we are about to overwrite
        self.manifest = None
        for _ in range(3):
            dl = self._download(v, manifest)
            if not dl.stale:
                break
            log.warning("%s: a source of v%d overwrote its copy mid-read; reading again", self.member, v)
        else:
            raise RuntimeError(f"v{v}: sources kept changing during the read")
        self.manifest = manifest
        self.stats = {"version": v, "bytes": manifest.total, "pull_s": time.perf_counter() - t0,
                      "sources": dl.sources, "source_failures": dl.failures}
        return manifest

    def _ensure_arena(self, total: int) -> None:
        if self.arena is not None and self.arena.numel() >= total:
            return
        if self.arena is not None:
            self.t.unregister(self.arena)
        self.arena = torch.empty(total, dtype=torch.uint8, device=self.device, pin_memory=self.pin)
        _stream_sync(self.arena)                    # the previous user of this memory must be done
        self.t.register(self.arena)

    def _let_go(self, dl: _Download) -> None:
        """Release the current assignment; a stale answer marks the download."""
        if dl.source is None:
            return
        r = self.reg.release(version=dl.version, source=dl.source["member"], member=self.member)
        dl.stale |= bool((r or {}).get("stale"))
        dl.source = None

    def _take_source(self, dl: _Download) -> None:
        dl.source = self.reg.assign(version=dl.version, member=self.member, exclude=sorted(dl.excluded))
        if dl.source is None:
            raise RuntimeError(f"no source holds version {dl.version}")
        dl.sources.append(dl.source["member"])

    def _source_failed(self, dl: _Download, err: TransferError) -> None:
        name = dl.source["member"]
        dl.next_chunk += getattr(err, "done", 0)        # the chunks before the failure did arrive
        dl.failures += 1
        log.warning("%s: read of v%d from %s failed (%s); switching source", self.member, dl.version, name, err)
        self.reg.report_failure(version=dl.version, source=name, reporter=self.member)
        self._let_go(dl)
        if name != PUBLISHER:
            dl.excluded.add(name)
        if dl.failures > self.max_fail:
            raise err

    def _download(self, version: int, manifest: WeightManifest) -> _Download:
        self._ensure_arena(manifest.total)
        dl = _Download(version, manifest.total, self.chunk)
        try:
            while not dl.finished:
                if dl.source is None:
                    self._take_source(dl)
                try:
                    self.t.read_window(dl.source["url"], dl.remaining_ops(), self.arena, self.window)
                    dl.next_chunk = len(dl.offsets)
                except TransferError as e:
                    self._source_failed(dl, e)
        except BaseException:
            try:
                self._let_go(dl)
            except Exception:  # noqa: BLE001
                pass
            raise
        self._let_go(dl)
        return dl

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
        manifest = self.pull(version)
        t0 = time.perf_counter()
        apply(self.tensors())
        _stream_sync(self.arena)
        self.stats["apply_s"] = time.perf_counter() - t0
        self.commit(manifest.version)
        return self.stats

    def close(self, leave: bool = True) -> None:
        self._stop.set()
        if leave:
            try:
                self.reg.leave(member=self.member)
            except Exception:  # noqa: BLE001
                pass
