"""Weight registry: the control plane of elastic weight sync.

The registry knows

* the latest published version and its manifest;
* the members (rollout engines): alive while they heartbeat within the TTL,
  and the version each has applied;
* for each of the last two versions, the *copies*: who holds a full copy
  (the publisher's arena, and members that keep theirs as relays), where to
  read it, and which readers are reading it right now.

``assign`` picks a copy for a reader: a copy below the fan-out limit if one
exists -- relays before the publisher, then the least busy -- else the least
busy copy, so the broadcast grows into a tree as members finish.
``retract`` / ``wait_idle`` protect a holder about to overwrite its copy: it
gets no new readers, and readers still on it when the bounded wait ends are
told on ``release`` that their bytes may be torn (``stale``) so they re-read.

:class:`RegistryServer` serves the method set over stdlib HTTP/JSON
(``POST /<method>`` with keyword arguments, reply ``{"result": ...}`` or
``{"error": ...}``); :class:`RegistryClient` is the matching client.
Method names, arguments and replies follow ``connex/rl/registry.py:24-284``
of the reference, so trainers and rollouts of either implementation
interoperate; the bookkeeping here is this module's own.
"""
from __future__ import annotations

import collections
import json
import threading
import time
import urllib.error
import urllib.request
from dataclasses import dataclass, field
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer
from typing import Dict, List, Optional, Set, Tuple

PUBLISHER = "trainer"

_METHODS = ("join", "heartbeat", "leave", "expire", "publish", "get_latest", "assign", "release",
            "report_failure", "retract", "wait_idle", "done", "status", "wait_all")


@dataclass
class _Copy:
    """A full copy of one version that readers may pull from."""

    url: str
    addr: int
    publisher: bool = False
    retiring: bool = False                  # about to be overwritten: no new readers
    readers: collections.Counter = field(default_factory=collections.Counter)

    @property
    def load(self) -> int:
        return sum(self.readers.values())


@dataclass
class _Member:
    url: str
    version: Optional[int] = None
    seen: float = field(default_factory=time.time)


class WeightRegistry:
    def __init__(self, fanout: int = 2, member_ttl_s: float = 10.0):
        self.fanout = fanout
        self.ttl = member_ttl_s
        self.lock = threading.Lock()
        self.cv = threading.Condition(self.lock)
        self.latest: Optional[dict] = None
        self.members: Dict[str, _Member] = {}
        self.holders: Dict[int, Dict[str, _Copy]] = {}      # version -> holder -> copy
        self.stale: Set[Tuple[str, int, str]] = set()       # (reader, version, source) with torn bytes
        self.events: collections.deque = collections.deque(maxlen=1000)

    def _log(self, kind, member, detail=None) -> None:
        self.events.append((time.time(), kind, member, detail))

    def _changed(self) -> None:
        self.cv.notify_all()

    # ------------------------------------------------------------- members
    def join(self, member, url=""):
        with self.cv:
            self.members[member] = _Member(url)
            self._log("join", member)
            return {"latest": self.latest["version"] if self.latest else None}

    def heartbeat(self, member):
        with self.cv:
            m = self.members.get(member)
            if m is not None:
                m.seen = time.time()
            return {"ok": m is not None}

    def leave(self, member, reason="leave"):
        with self.cv:
            self.members.pop(member, None)
            for copies in self.holders.values():
                copies.pop(member, None)                     # its copy is gone
                for c in copies.values():
                    c.readers.pop(member, None)              # its reads give their load back
            self.stale = {s for s in self.stale if s[0] != member}
            self._log(reason, member)
            self._changed()
            return {"ok": True}

    def expire(self):
        cutoff = time.time() - self.ttl
        with self.cv:
            gone = [name for name, m in self.members.items() if m.seen < cutoff]
        for name in gone:
            self.leave(name, "expired")
        return gone

    # ------------------------------------------------------------ versions
    def publish(self, version, manifest, url, addr):
        with self.cv:
            if self.latest and version <= self.latest["version"]:
                raise ValueError(f"version {version} <= latest {self.latest['version']}")
            self.latest = {"version": version, "manifest": manifest}
            self.holders[version] = {PUBLISHER: _Copy(url, addr, publisher=True)}
            for old in [v for v in self.holders if v < version - 1]:
                del self.holders[old]                        # keep the last two versions
            self._log("publish", PUBLISHER, version)
            self._changed()
            return {"ok": True}

    def get_latest(self, wait_newer_than=None, timeout=0.0):
        with self.cv:
            if wait_newer_than is not None:
                self.cv.wait_for(lambda: self.latest is not None and self.latest["version"] > wait_newer_than,
                                 timeout=timeout)
            return self.latest

    def _preference(self, copy: _Copy):
        """Sort key of a copy for a new reader (smaller is better)."""
        load = copy.load
        if load < self.fanout:
            return 0, 0, copy.publisher, load
        return 1, load, copy.publisher, load

    def assign(self, version, member, exclude=()):
        with self.cv:
            options = [(name, c) for name, c in self.holders.get(version, {}).items()
                       if name != member and name not in exclude and not c.retiring]
            if not options:
                return None
            name, copy = min(options, key=lambda nc: self._preference(nc[1]))
            copy.readers[member] += 1
            return {"member": name, "url": copy.url, "addr": copy.addr}

    def release(self, version, source, member=None):
        with self.cv:
            copy = self.holders.get(version, {}).get(source)
            if member is None:
                # an anonymous release: give back one unit of load
                if copy is not None and copy.readers:
                    reader = next(iter(copy.readers))
                    copy.readers[reader] -= 1
                    if copy.readers[reader] <= 0:
                        del copy.readers[reader]
                self._changed()
                return {"ok": True}
            if copy is not None and copy.readers.get(member, 0) > 0:
                copy.readers[member] -= 1
                if copy.readers[member] <= 0:
                    del copy.readers[member]
                self._changed()
            # the copy may be gone already (retired / older than the last two
            # versions): a reader it was invalidated under still learns so
            if (member, version, source) in self.stale:
                self.stale.discard((member, version, source))
                return {"ok": True, "stale": True}
            return {"ok": True}

    def invalidate(self, version, source) -> None:
        """Readers now on ``source`` (of ``version``, or any version when None)
        will hear on release that their bytes may be torn.  Lock held."""
        for v, copies in self.holders.items():
            copy = copies.get(source)
            if copy is None or (version is not None and v != version):
                continue
            self.stale.update((reader, v, source) for reader in copy.readers)

    def report_failure(self, version, source, reporter):
        with self.cv:
            copies = self.holders.get(version, {})
            if source in copies and not copies[source].publisher:
                del copies[source]
            self._log("source_failed", source, {"version": version, "by": reporter})
            self._changed()
            return {"ok": True}

    def _busy(self, member, version=None) -> int:
        return sum(c[member].load for v, c in self.holders.items()
                   if member in c and (version is None or v == version))

    def retract(self, member, timeout=5.0):
        """``member`` is about to overwrite its copies: wait (bounded) for its
        readers, mark the rest stale, and drop the copies."""
        with self.cv:
            if not self.cv.wait_for(lambda: self._busy(member) == 0, timeout=timeout):
                self.invalidate(None, member)
            for copies in self.holders.values():
                copies.pop(member, None)
            return {"ok": True}

    def wait_idle(self, version, member=PUBLISHER, timeout=5.0, retire=False):
        with self.cv:
            copy = self.holders.get(version, {}).get(member)
            if retire and copy is not None:
                copy.retiring = True
            idle = self.cv.wait_for(lambda: self._busy(member, version) == 0, timeout=timeout)
            if not idle:
                self.invalidate(version, member)
            if retire:
                self.holders.get(version, {}).pop(member, None)
            return {"ok": bool(idle)}

    def done(self, version, member, url, addr, hold=True):
        """``member`` applied ``version``; with ``hold`` it keeps the copy as a relay."""
        with self.cv:
            m = self.members.setdefault(member, _Member(url))
            m.version, m.seen = version, time.time()
            if hold and version in self.holders:
                self.holders[version][member] = _Copy(url, addr)
            self._log("applied", member, version)
            self._changed()
            return {"ok": True}

    def status(self):
        with self.cv:
            return {"latest": self.latest["version"] if self.latest else None,
                    "members": {name: m.version for name, m in self.members.items()},
                    "holders": {str(v): {name: c.load for name, c in copies.items()}
                                for v, copies in self.holders.items()}}

    def wait_all(self, version, timeout=60.0):
        with self.cv:
            return self.cv.wait_for(lambda: all(m.version == version for m in self.members.values()),
                                    timeout=timeout)


class _Handler(BaseHTTPRequestHandler):
    registry: WeightRegistry

    def log_message(self, *args):
        return None

    def _reply(self, code: int, body: dict) -> None:
        data = json.dumps(body).encode()
        self.send_response(code)
        self.send_header("Content-Length", str(len(data)))
        self.end_headers()
        self.wfile.write(data)

    def do_POST(self):
        method = self.path.strip("/")
        try:
            kwargs = json.loads(self.rfile.read(int(self.headers.get("Content-Length") or 0)) or b"{}")
            if method not in _METHODS:
                raise KeyError(method)
            self._reply(200, {"result": getattr(self.registry, method)(**kwargs)})
        except Exception as e:  # noqa: BLE001 - reported to the caller
            self._reply(400, {"error": f"{type(e).__name__}: {e}"})


class RegistryServer:
    """Serves a :class:`WeightRegistry` over HTTP and expires silent members."""

    def __init__(self, registry: Optional[WeightRegistry] = None, host: str = "0.0.0.0", port: int = 0,
                 expire_interval: float = 1.0):
        self.reg = registry or WeightRegistry()
        handler = type("RegistryHandler", (_Handler,), {"registry": self.reg})
        self.httpd = ThreadingHTTPServer((host, port), handler)
        self.httpd.daemon_threads = True
        self.port = self.httpd.server_address[1]
        self._stop = threading.Event()
        for target in (self.httpd.serve_forever, lambda: self._expire_loop(expire_interval)):
            threading.Thread(target=target, daemon=True).start()

    def _expire_loop(self, every: float) -> None:
        while not self._stop.wait(every):
            self.reg.expire()

    def close(self) -> None:
        self._stop.set()
        self.httpd.shutdown()
        self.httpd.server_close()


class RegistryClient:
    """The :class:`WeightRegistry` methods over HTTP (environment proxies ignored)."""

    def __init__(self, url: str, timeout: float = 120.0):
        self.url = url.rstrip("/")
        self.timeout = timeout
        self._opener = urllib.request.build_opener(urllib.request.ProxyHandler({}))

    def _post(self, method: str, kwargs: dict):
        req = urllib.request.Request(f"{self.url}/{method}", data=json.dumps(kwargs).encode(),
                                     headers={"Content-Type": "application/json"})
        try:
            with self._opener.open(req, timeout=self.timeout) as r:
                return json.loads(r.read())["result"]
        except urllib.error.HTTPError as e:
            raw = e.read()
            try:
                message = json.loads(raw).get("error")
            except ValueError:
                message = f"HTTP {e.code}: {raw[:200]!r}"
            raise RuntimeError(message) from None


def _remote(method: str):
    def call(self, **kwargs):
        return self._post(method, kwargs)
    call.__name__ = method
    call.__doc__ = f"``WeightRegistry.{method}`` on the server."
    return call


for _m in _METHODS:
    setattr(RegistryClient, _m, _remote(_m))
del _m
