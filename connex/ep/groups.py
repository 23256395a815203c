"""Replica-level recovery of EP groups.

The ranks of one EP group run collectives every step, so losing one rank
stops the whole group; recovery therefore happens one level up, where each
EP group is a mobile endpoint (its API URL) behind the resume proxy.

:class:`EPGroupSupervisor` judges every group that is ``up`` on each tick:

* its launcher process exited -> failed at once;
* one of its rank processes exited (or is a zombie) -> failed at once;
* ``fail_after`` health probes in a row failed -> failed.

A failed group leaves the endpoints file (which the proxy re-reads), is
rebuilt by its ``restart`` callback on a worker thread, and rejoins the file
once it answers its health probe again (``on_rejoin`` then runs).  Every
transition is recorded in ``events`` with timings.

:class:`RankDeathWatcher` fails a group as soon as the transfer engine
reports one of its ranks dead (a reset socket of a dead process, wherever
it ran) -- faster than any probe.

Behavioural parity: ``connex/ep/groups.py:53-267`` of the reference.
"""
from __future__ import annotations

import logging
import os
import threading
import time
import urllib.request
from typing import Callable, Dict, List, Optional, Tuple

log = logging.getLogger("connex.ep")

DEFAULT_PROBE_TIMEOUT = 3.0
UP, DOWN, REBUILDING = "up", "down", "rebuilding"


def _healthy(url: str, timeout: Optional[float] = None, path: Optional[str] = None) -> bool:
    """GET ``url + path`` (no proxies) answers 200 within ``timeout``."""
    if timeout is None:
        timeout = float(os.environ.get("CONNEX_EP_PROBE_TIMEOUT", DEFAULT_PROBE_TIMEOUT))
    if path is None:
        path = os.environ.get("CONNEX_EP_PROBE_PATH", "/health")
    target = f"{url.rstrip('/')}/{path.lstrip('/')}"
    try:
        with urllib.request.build_opener(urllib.request.ProxyHandler({})).open(target, timeout=timeout) as r:
            return r.status == 200
    except Exception:  # noqa: BLE001 - any failure is "not healthy"
        return False


def pid_alive(pid: int) -> bool:
    """The process runs and is not a zombie (a killed, unreaped rank still
    answers ``kill(pid, 0)``)."""
    try:
        with open(f"/proc/{pid}/stat") as f:
            state = f.read().rsplit(")", 1)[1].split()[0]
        return state not in ("Z", "X")
    except (OSError, IndexError):
        pass
    try:
        os.kill(pid, 0)
    except OSError:
        return False
    return True


class EPGroup:
    """One EP group: its API URL, how to rebuild it (``restart() -> proc``),
    its launcher process and (optionally) a callable listing its rank PIDs."""

    def __init__(self, name: str, url: str, restart: Optional[Callable] = None, proc=None,
                 rank_pids: Optional[Callable] = None, on_rejoin: Optional[Callable] = None):
        self.name = name
        self.url = url.rstrip("/")
        self.restart = restart
        self.proc = proc
        self.rank_pids = rank_pids
        self.on_rejoin = on_rejoin
        self.state = UP
        self.fails = 0                     # consecutive failed probes
        self._pids: Optional[List[int]] = None

    def launcher_exited(self) -> bool:
        return self.proc is not None and self.proc.poll() is not None

    def ranks(self) -> Optional[List[int]]:
        """The rank PIDs (asked once per incarnation)."""
        if self.rank_pids is not None and not self._pids:
            try:
                self._pids = list(self.rank_pids() or [])
            except Exception:  # noqa: BLE001 - not known yet
                self._pids = None
        return self._pids

    def reset(self) -> None:
        self.state, self.fails, self._pids = UP, 0, None


class EPGroupSupervisor:
    def __init__(self, groups, endpoints_file: str, probe_s: float = 0.5, fail_after: int = 2,
                 start_timeout: float = 600.0, probe: Optional[Callable[[str], bool]] = None,
                 probe_timeout: Optional[float] = None, probe_path: Optional[str] = None):
        self.groups: Dict[str, EPGroup] = {g.name: g for g in groups}
        self.file = endpoints_file
        self.probe_s = probe_s
        self.fail_after = fail_after
        self.start_timeout = start_timeout
        self.probe = probe or (lambda url: _healthy(url, probe_timeout, probe_path))
        self.events: List[dict] = []
        self._lock = threading.Lock()
        self._stop = threading.Event()
        self._th: Optional[threading.Thread] = None
        self.write_endpoints()

    def _event(self, kind: str, group: str, **kw) -> None:
        self.events.append({"t": time.time(), "kind": kind, "group": group, **kw})
        log.info("ep-group %s %s %s", group, kind, kw)

    def write_endpoints(self) -> None:
        """Atomically rewrite the file with the URLs of the groups that are up."""
        urls = [g.url for g in self.groups.values() if g.state == UP]
        tmp = self.file + ".tmp"
        with open(tmp, "w") as f:
            f.write("\n".join(urls) + "\n")
        os.replace(tmp, self.file)

    def _verdict(self, g: EPGroup) -> Optional[str]:
        """Why ``g`` counts as failed now, or None."""
        if g.launcher_exited():
            return "process exited"
        pids = g.ranks()
        if pids and not all(pid_alive(p) for p in pids):
            return "rank process exited"
        g.fails = 0 if self.probe(g.url) else g.fails + 1
        return "health probe" if g.fails >= self.fail_after else None

    def check_once(self) -> None:
        for g in [g for g in self.groups.values() if g.state == UP]:
            why = self._verdict(g)
            if why is not None:
                self.on_failure(g, why)

    def on_failure(self, g: EPGroup, why: str) -> None:
        with self._lock:
            if g.state != UP:
                return                          # already handled
            g.state = DOWN
            self.write_endpoints()
            self._event("down", g.name, why=why)
        if g.restart is not None:
            threading.Thread(target=self._rebuild, args=(g,), daemon=True).start()

    def _serving_again(self, g: EPGroup, t0: float) -> Tuple[bool, str]:
        while time.time() - t0 < self.start_timeout and not self._stop.is_set():
            if g.launcher_exited():
                return False, "exited during start"
            if self.probe(g.url):
                return True, ""
            time.sleep(self.probe_s)
        return False, "timeout"

    def _rebuild(self, g: EPGroup) -> None:
        t0 = time.time()
        g.state = REBUILDING
        self._event("rebuild-start", g.name)
        try:
            if g.proc is not None and g.proc.poll() is None:
                g.proc.kill()
            g.proc = g.restart()
        except Exception as ex:  # noqa: BLE001
            self._event("rebuild-failed", g.name, error=repr(ex))
            g.state = DOWN
            return
        ok, why = self._serving_again(g, t0)
        if not ok:
            self._event("rebuild-failed", g.name, error=why)
            g.state = DOWN
            return
        with self._lock:
            g.reset()
            self.write_endpoints()
        self._event("rejoin", g.name, rebuild_s=time.time() - t0)
        if g.on_rejoin is not None:
            try:
                g.on_rejoin(g)
            except Exception as ex:  # noqa: BLE001
                self._event("rejoin-hook-failed", g.name, error=repr(ex))

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
    """Fails a rank's group when the transfer engine reports that rank dead.
    Ranks are known by their engine URL ``ip:port#connex-ep|0|<rank>|<group>``."""

    def __init__(self, supervisor: EPGroupSupervisor, engine=None):
        from connex.pd.group import EventPump, GroupFailureTracker
        if engine is None:
            from connex_b200.engine import Engine
            engine = Engine("connex-ep-watch", 0, 0, 0, listen_ip="127.0.0.1")
        self.sup = supervisor
        self.engine = engine
        self.tracker = GroupFailureTracker("connex-ep", [0])
        self.groups: Dict[tuple, str] = {}
        self.reports: List[tuple] = []
        self._pump = EventPump(engine, self.handle, name="connex-ep-rank-watch")

    @staticmethod
    def identity(url: str) -> tuple:
        model, stage, shard, replica = url.split("#", 1)[1].split("|")
        return model, int(stage), int(shard), int(replica)

    def watch(self, group_name: str, urls) -> None:
        for u in urls:
            self.groups[self.identity(u)] = group_name
            self.engine.connect(u)

    def handle(self, ev: dict) -> Optional[str]:
        lid = self.tracker.on_event(ev)
        if lid is None:
            return None
        key = (lid.model_name, lid.stage_idx, lid.shard_idx, lid.replica_idx)
        g = self.sup.groups.get(self.groups.get(key, ""))
        if g is None or g.state != UP:
            return None
        self.reports.append((time.time(), g.name, key))
        self.sup.on_failure(g, f"rank {lid.shard_idx} died (transport)")
        return g.name

    def start(self) -> None:
        self._pump.start()

    def stop(self) -> None:
        self._pump.stop()
