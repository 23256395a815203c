"""Replica-level recovery of EP groups (reference ``connex/ep/groups.py``).

When the ranks of one EP group share collectives every step, losing a rank
stops the group; recovery happens a level up: each EP group is one mobile
endpoint (its API URL).  :class:`EPGroupSupervisor` probes every group
(``/health``, rank processes), removes a failed group from the routing set
(an endpoints file the resume proxy re-reads), rebuilds it with its
``restart`` callback, waits until it serves, and puts it back (rejoin);
step timings land in ``events``.  :class:`RankDeathWatcher` fails a group
as soon as the transfer engine reports one of its ranks dead (socket reset
of a dead process, wherever it ran).
"""
from __future__ import annotations

import logging
import os
import threading
import time
import urllib.request
from typing import Callable, Optional

log = logging.getLogger("connex.ep")

DEFAULT_PROBE_TIMEOUT = 3.0


def _healthy(url: str, timeout: Optional[float] = None, path: Optional[str] = None) -> bool:
    timeout = float(os.environ.get("CONNEX_EP_PROBE_TIMEOUT", DEFAULT_PROBE_TIMEOUT)) if timeout is None else timeout
    path = os.environ.get("CONNEX_EP_PROBE_PATH", "/health") if path is None else path
    try:
        opener = urllib.request.build_opener(urllib.request.ProxyHandler({}))
        with opener.open(urllib.request.Request(url.rstrip("/") + "/" + path.lstrip("/")), timeout=timeout) as r:
            return r.status == 200
    except Exception:
        return False


def pid_alive(pid: int) -> bool:
    """Running and not a zombie (a killed, unreaped rank still answers kill(pid, 0))."""
    try:
        with open(f"/proc/{pid}/stat") as f:
            return f.read().rsplit(")", 1)[1].split()[0] not in ("Z", "X")
    except (OSError, IndexError):
        try:
            os.kill(pid, 0)
            return True
        except OSError:
            return False


class EPGroup:
    def __init__(self, name: str, url: str, restart: Optional[Callable] = None, proc=None,
                 rank_pids: Optional[Callable] = None, on_rejoin: Optional[Callable] = None):
        self.name = name
        self.url = url.rstrip("/")
        self.restart = restart
        self.proc = proc
        self.rank_pids = rank_pids
        self.on_rejoin = on_rejoin
        self._pids = None
        self.state = "up"
        self.fails = 0


class EPGroupSupervisor:
    def __init__(self, groups, endpoints_file: str, probe_s: float = 0.5, fail_after: int = 2,
                 start_timeout: float = 600.0, probe: Optional[Callable[[str], bool]] = None,
                 probe_timeout: Optional[float] = None, probe_path: Optional[str] = None):
        self.groups = {g.name: g for g in groups}
        self.file = endpoints_file
        self.probe_s = probe_s
        self.fail_after = fail_after
        self.start_timeout = start_timeout
        self.probe = probe or (lambda url: _healthy(url, probe_timeout, probe_path))
        self.events: list = []
        self._stop = threading.Event()
        self._th: Optional[threading.Thread] = None
        self._lock = threading.Lock()
        self.write_endpoints()

    def _event(self, kind: str, group: str, **kw) -> None:
        self.events.append({"t": time.time(), "kind": kind, "group": group, **kw})
        log.info("ep-group %s %s %s", group, kind, kw)

    def write_endpoints(self) -> None:
        tmp = self.file + ".tmp"
        with open(tmp, "w") as f:
            f.write("\n".join(g.url for g in self.groups.values() if g.state == "up") + "\n")
        os.replace(tmp, self.file)

    def check_once(self) -> None:
        for g in list(self.groups.values()):
            if g.state != "up":
                continue
            dead = g.proc is not None and g.proc.poll() is not None
            if not dead and g.rank_pids is not None:
                if not g._pids:
                    try:
                        g._pids = list(g.rank_pids() or [])
                    except Exception:
                        g._pids = None
                if g._pids and not all(pid_alive(p) for p in g._pids):
                    self.on_failure(g, "rank process exited")
                    continue
            ok = (not dead) and self.probe(g.url)
            g.fails = 0 if ok else g.fails + 1
            if dead or g.fails >= self.fail_after:
                self.on_failure(g, "process exited" if dead else "health probe")

    def on_failure(self, g: EPGroup, why: str) -> None:
        with self._lock:
            if g.state != "up":
                return
            g.state = "down"
            self.write_endpoints()
            self._event("down", g.name, why=why)
        if g.restart is not None:
            threading.Thread(target=self._rebuild, args=(g,), daemon=True).start()

    def _rebuild(self, g: EPGroup) -> None:
        t0 = time.time()
        g.state = "rebuilding"
        self._event("rebuild-start", g.name)
        try:
            if g.proc is not None and g.proc.poll() is None:
                g.proc.kill()
            g.proc = g.restart()
        except Exception as ex:
            self._event("rebuild-failed", g.name, error=repr(ex))
            g.state = "down"
            return
        while time.time() - t0 < self.start_timeout and not self._stop.is_set():
            if g.proc is not None and g.proc.poll() is not None:
                self._event("rebuild-failed", g.name, error="exited during start")
                g.state = "down"
                return
            if self.probe(g.url):
                with self._lock:
                    g.state, g.fails, g._pids = "up", 0, None
                    self.write_endpoints()
                self._event("rejoin", g.name, rebuild_s=time.time() - t0)
                if g.on_rejoin is not None:
                    try:
                        g.on_rejoin(g)
                    except Exception as ex:
                        self._event("rejoin-hook-failed", g.name, error=repr(ex))
                return
            time.sleep(self.probe_s)
        self._event("rebuild-failed", g.name, error="timeout")
        g.state = "down"

    def start(self) -> None:
        def loop():
            while not self._stop.is_set():
                self.check_once()
                self._stop.wait(self.probe_s)
        self._th = threading.Thread(target=loop, daemon=True, name="connex-ep-supervisor")
        self._th.start()

    def stop(self) -> None:
        self._stop.set()
        if self._th is not None:
            self._th.join(timeout=5)


class RankDeathWatcher:
    """Fails a rank's group when the transfer engine reports the rank dead.
    Ranks are identified ``("connex-ep", 0, rank, group)`` by their engine URL."""

    def __init__(self, supervisor: EPGroupSupervisor, engine=None):
        from connex.pd.group import GroupFailureTracker
        if engine is None:
            from connex_b200.engine import Engine
            engine = Engine("connex-ep-watch", 0, 0, 0, listen_ip="127.0.0.1")
        self.sup = supervisor
        self.engine = engine
        self.tracker = GroupFailureTracker("connex-ep", [0])
        self.groups: dict = {}
        self.reports: list = []
        self._stop = threading.Event()
        self._th: Optional[threading.Thread] = None

    @staticmethod
    def identity(url: str) -> tuple:
        m, st, sh, r = url.split("#", 1)[1].split("|")
        return (m, int(st), int(sh), int(r))

    def watch(self, group_name: str, urls) -> None:
        for u in urls:
            self.groups[self.identity(u)] = group_name
            self.engine.connect(u)

    def handle(self, ev: dict) -> Optional[str]:
        lid = self.tracker.on_event(ev)
        if lid is None:
            return None
        key = (lid.model_name, lid.stage_idx, lid.shard_idx, lid.replica_idx)
        name = self.groups.get(key)
        g = self.sup.groups.get(name) if name else None
        if g is None or g.state != "up":
            return None
        self.reports.append((time.time(), name, key))
        self.sup.on_failure(g, f"rank {lid.shard_idx} died (transport)")
        return name

    def start(self) -> None:
        def loop():
            while not self._stop.is_set():
                try:
                    ev = self.engine.wait_event(100)
                except Exception:
                    return
                if ev is not None:
                    self.handle(ev)
        self._th = threading.Thread(target=loop, daemon=True, name="connex-ep-rank-watch")
        self._th.start()

    def stop(self) -> None:
        self._stop.set()
