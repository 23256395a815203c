"""Weight registry: the control plane of elastic weight sync (reference
``connex/rl/registry.py:24-284``).

Knows the latest published version and its manifest, which members
(rollout engines) are alive (TTL) and at which version, and who holds a
full copy of each version (the last two versions are kept).  ``assign``
hands a reader a source with spare fan-out, so the broadcast becomes a tree
that grows as members finish (the publisher serves only when it has spare
fan-out too).  ``retract`` / ``wait_idle`` guard a holder that is about to
overwrite its copy: readers still assigned to it when the bounded wait
expires are told on ``release`` that their bytes may be torn (``stale``).

:class:`RegistryServer` serves the same method set over stdlib HTTP/JSON
(``POST /<method>`` with keyword arguments; reply ``{"result": ...}`` or
``{"error": ...}``) and :class:`RegistryClient` calls it.
"""
from __future__ import annotations

import json
import threading
import time
import urllib.error
import urllib.request
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer
from typing import Optional

PUBLISHER = "trainer"

_METHODS = {"join", "heartbeat", "leave", "expire", "publish", "get_latest", "assign", "release", "report_failure",
            "retract", "wait_idle", "done", "status", "wait_all"}


class WeightRegistry:
    def __init__(self, fanout: int = 2, member_ttl_s: float = 10.0):
        self.fanout = fanout
        self.ttl = member_ttl_s
        self.lock = threading.Lock()
        self.cv = threading.Condition(self.lock)
        self.latest: Optional[dict] = None
        self.holders: dict = {}    # version -> {member: {url, addr, load, publisher}}
        self.members: dict = {}    # member -> {url, version, last_seen}
        self.events: list = []
        self.reading: dict = {}    # reader -> [(version, source)]
        self.stale: set = set()    # (reader, version, source)

    def _ev(self, kind, member, detail=None):
        self.events.append((time.time(), kind, member, detail))
        del self.events[:-1000]

    # ---------------------------------------------------------- membership
    def join(self, member, url=""):
        with self.lock:
            self.members[member] = {"url": url, "version": None, "last_seen": time.time()}
            self._ev("join", member)
            return {"latest": self.latest["version"] if self.latest else None}

    def heartbeat(self, member):
        with self.lock:
            if member in self.members:
                self.members[member]["last_seen"] = time.time()
                return {"ok": True}
            return {"ok": False}

    def leave(self, member, reason="leave"):
        with self.cv:
            self.members.pop(member, None)
            for version, source in self.reading.pop(member, []):  # give its load back
                self._release(version, source)
            self.stale = {x for x in self.stale if x[0] != member}
            for hs in self.holders.values():
                hs.pop(member, None)
            self._ev(reason, member)
            self.cv.notify_all()
            return {"ok": True}

    def expire(self):
        now = time.time()
        with self.lock:
            dead = [m for m, i in self.members.items() if now - i["last_seen"] > self.ttl]
        for m in dead:
            self.leave(m, "expired")
        return dead

    # ------------------------------------------------------------ versions
    def publish(self, version, manifest, url, addr):
        with self.cv:
            if self.latest and version <= self.latest["version"]:
                raise ValueError(f"version {version} <= latest {self.latest['version']}")
            self.latest = {"version": version, "manifest": manifest}
            self.holders[version] = {PUBLISHER: {"url": url, "addr": addr, "load": 0, "publisher": True}}
            for v in [v for v in self.holders if v < version - 1]:
                del self.holders[v]
            self._ev("publish", PUBLISHER, version)
            self.cv.notify_all()
            return {"ok": True}

    def get_latest(self, wait_newer_than=None, timeout=0.0):
        with self.cv:
            if wait_newer_than is not None:
                self.cv.wait_for(lambda: self.latest and self.latest["version"] > wait_newer_than, timeout=timeout)
            return self.latest

    def assign(self, version, member, exclude=()):
        with self.lock:
            hs = {m: h for m, h in self.holders.get(version, {}).items()
                  if m != member and m not in exclude and not h.get("retiring")}
            if not hs:
                return None

            def key(item):
                _, h = item
                full = h["load"] >= self.fanout
                return (full, h["load"] if full else 0, h["publisher"], h["load"])
            m, h = min(hs.items(), key=key)
            h["load"] += 1
            self.reading.setdefault(member, []).append((version, m))
            return {"member": m, "url": h["url"], "addr": h["addr"]}

    def _release(self, version, source):
        h = self.holders.get(version, {}).get(source)
        if h and h["load"] > 0:
            h["load"] -= 1

    def release(self, version, source, member=None):
        with self.cv:
            if member is not None:
                rs = self.reading.get(member, [])
                if (version, source) not in rs:
                    return {"ok": True}
                rs.remove((version, source))
                if not rs:
                    self.reading.pop(member, None)
            self._release(version, source)
            self.cv.notify_all()
            if member is not None and (member, version, source) in self.stale:
                self.stale.discard((member, version, source))
                return {"ok": True, "stale": True}
            return {"ok": True}

    def _invalidate(self, version, source):
        for reader, rs in self.reading.items():
            for v, src in rs:
                if src == source and (version is None or v == version):
                    self.stale.add((reader, v, src))

    def report_failure(self, version, source, reporter):
        with self.cv:
            h = self.holders.get(version, {})
            if source in h and not h[source]["publisher"]:
                del h[source]
            self._ev("source_failed", source, {"version": version, "by": reporter})
            self.cv.notify_all()
            return {"ok": True}

    def retract(self, member, timeout=5.0):
        with self.cv:
            def busy():
                return sum(h[member]["load"] for h in self.holders.values() if member in h)
            if not self.cv.wait_for(lambda: busy() == 0, timeout=timeout):
                self._invalidate(None, member)
            for hs in self.holders.values():
                hs.pop(member, None)
            return {"ok": True}

    def wait_idle(self, version, member=PUBLISHER, timeout=5.0, retire=False):
        with self.cv:
            h = self.holders.get(version, {}).get(member)
            if retire and h is not None:
                h["retiring"] = True       # the copy is about to be overwritten: no new readers
            ok = self.cv.wait_for(lambda: self.holders.get(version, {}).get(member, {"load": 0})["load"] == 0,
                                  timeout=timeout)
            if not ok:
                self._invalidate(version, member)
            if retire:
                self.holders.get(version, {}).pop(member, None)
            return {"ok": bool(ok)}

    def done(self, version, member, url, addr, hold=True):
        with self.cv:
            if member not in self.members:
                self.members[member] = {"url": url, "version": None, "last_seen": time.time()}
            self.members[member].update(version=version, last_seen=time.time())
            if hold and version in self.holders:
                self.holders[version][member] = {"url": url, "addr": addr, "load": 0, "publisher": False}
            self._ev("applied", member, version)
            self.cv.notify_all()
            return {"ok": True}

    def status(self):
        with self.lock:
            return {"latest": self.latest["version"] if self.latest else None,
                    "members": {m: i["version"] for m, i in self.members.items()},
                    "holders": {str(v): {m: h["load"] for m, h in hs.items()} for v, hs in self.holders.items()}}

    def wait_all(self, version, timeout=60.0):
        with self.cv:
            return self.cv.wait_for(lambda: all(i["version"] == version for i in self.members.values()),
                                    timeout=timeout)


class RegistryServer:
    def __init__(self, registry: Optional[WeightRegistry] = None, host: str = "0.0.0.0", port: int = 0,
                 expire_interval: float = 1.0):
        self.reg = registry or WeightRegistry()
        reg = self.reg

        class Handler(BaseHTTPRequestHandler):
            def log_message(self, *a):
                pass

            def do_POST(self):
                name = self.path.strip("/")
                n = int(self.headers.get("Content-Length") or 0)
                try:
                    body = json.loads(self.rfile.read(n) or b"{}")
                    if name not in _METHODS:
                        raise KeyError(name)
                    out, code = {"result": getattr(reg, name)(**body)}, 200
                except Exception as e:
                    out, code = {"error": f"{type(e).__name__}: {e}"}, 400
                data = json.dumps(out).encode()
                self.send_response(code)
                self.send_header("Content-Length", str(len(data)))
                self.end_headers()
                self.wfile.write(data)

        self.httpd = ThreadingHTTPServer((host, port), Handler)
        self.httpd.daemon_threads = True
        self.port = self.httpd.server_address[1]
        self._stop = threading.Event()
        self._threads = [threading.Thread(target=self.httpd.serve_forever, daemon=True),
                         threading.Thread(target=self._expire_loop, args=(expire_interval,), daemon=True)]
        for t in self._threads:
            t.start()

    def _expire_loop(self, every: float) -> None:
        while not self._stop.wait(every):
            self.reg.expire()

    def close(self) -> None:
        self._stop.set()
        self.httpd.shutdown()
        self.httpd.server_close()


class RegistryClient:
    """Same methods as :class:`WeightRegistry`, over HTTP (no env proxies)."""

    def __init__(self, url: str, timeout: float = 120.0):
        self.url = url.rstrip("/")
        self.timeout = timeout
        self._open = urllib.request.build_opener(urllib.request.ProxyHandler({})).open

    def __getattr__(self, name):
        if name not in _METHODS:
            raise AttributeError(name)

        def call(**kw):
            req = urllib.request.Request(f"{self.url}/{name}", data=json.dumps(kw).encode(),
                                         headers={"Content-Type": "application/json"})
            try:
                with self._open(req, timeout=self.timeout) as r:
                    return json.loads(r.read())["result"]
            except urllib.error.HTTPError as e:
                body = e.read()
                try:
                    msg = json.loads(body).get("error")
                except ValueError:
                    msg = f"HTTP {e.code}: {body[:200]!r}"
                raise RuntimeError(msg) from None
        return call
