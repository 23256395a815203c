"""Liveness protocol of an elastic pipeline: control messages between stage 0
and the stage replicas, carried by the PP endpoints' own sockets.

Failure detection has three tiers (fastest first):

1. **transport events** -- the native engine reports a peer's socket reset
   or heartbeat loss within milliseconds; a confirmed death of the
   downstream replica fails over at once
   (:meth:`connex.pp.endpoint.PipelineEndpoint.watch_peers`);
2. **membership** -- a missed lease makes a peer suspect and a TCP probe
   decides (the endpoint's membership handlers);
3. **the step watchdog** -- a stage that is alive but hung (a stuck GPU
   stream, a deadlocked worker) is found by its late step
   (:class:`ChainWatchdog`).

Messages (JSON, ``kind`` plus the sender's ``from`` / ``stage`` /
``replica``):

=========  ======================  ============================================
kind       direction               meaning
=========  ======================  ============================================
HELLO      stage 0 -> replica      "I route to you" (claims ownership)
HELLO_OK   replica -> stage 0      accepted; the replica is alive from now on
BUSY       replica -> stage 0      owned by another live stage 0: go elsewhere
READY      replica -> stage 0      (re)started and serving; answered by HELLO
DYING      replica -> stage 0      exiting: fail over now, do not wait
PING       stage 0 -> replica      liveness check of the route
PONG       replica -> stage 0      alive; ``done_seq`` (last step answered) and
                                   ``next`` (its own downstream address)
FAILOVER   stage 0 -> replica      fail over your downstream replica
=========  ======================  ============================================

A replica has one owner (a stage-0 instance) at a time; another stage 0's
HELLO is answered BUSY until the owner has been silent for ``takeover_s``
(no step, no PING), then it takes over.  A replica remembers the stage-0
instances that said HELLO in a small state file (:class:`HeadState`) and
announces READY to them after a restart, so it rejoins as a spare without
a scheduler restart.

Behavioural parity: the control protocol of
``connex/adapters/vllm/pp/executor.py:68-216,453-612`` and
``connex/adapters/vllm/pp/stage.py:52-130`` in the reference (HELLO / READY /
DYING / BUSY / PING, adaptive step timeout, pick-stuck, the false-failure
ping after a rejoin, the head-state file); here it serves this framework's
own stage runtime.
"""
from __future__ import annotations

import collections
import json
import logging
import os
import threading
import time
from dataclasses import dataclass
from typing import Callable, Deque, Dict, List, Optional, Sequence, Tuple

log = logging.getLogger("connex.pp.liveness")

HELLO, HELLO_OK, BUSY, READY, DYING = "HELLO", "HELLO_OK", "BUSY", "READY", "DYING"
PING, PONG, FAILOVER = "PING", "PONG", "FAILOVER"
REJOIN_GRACE_S = 30.0      # a failure event this soon after HELLO_OK is checked by a PING first


class HeadState:
    """The stage-0 addresses a replica has served (the last ``keep``), kept in
    a JSON file that survives a restart of the replica's process."""

    def __init__(self, path: str, keep: int = 8):
        self.path, self.keep = path, keep
        self.heads: List[str] = self._load()

    def _load(self) -> List[str]:
        try:
            with open(self.path) as f:
                return [h for h in json.load(f) if isinstance(h, str)][-self.keep:]
        except (OSError, ValueError):
            return []

    def remember(self, head: str) -> None:
        if not head or head in self.heads:
            return
        self.heads = (self.heads + [head])[-self.keep:]
        tmp = f"{self.path}.{os.getpid()}"
        try:
            with open(tmp, "w") as f:
                json.dump(self.heads, f)
            os.replace(tmp, self.path)
        except OSError as e:
            log.warning("cannot keep stage-0 addresses in %s: %s", self.path, e)


def default_state_dir() -> str:
    return os.getenv("CONNEX_PP_STATE_DIR") or ("/dev/shm" if os.path.isdir("/dev/shm") else "/tmp")


class StageResponder:
    """Replica side of the protocol for one stage endpoint (stages 1..)."""

    def __init__(self, ep, state_dir: Optional[str] = None, takeover_s: float = 10.0):
        self.ep = ep
        self.takeover_s = takeover_s
        self.owner: Optional[str] = None
        self._owner_seen = 0.0
        path = os.path.join(state_dir or default_state_dir(),
                            f"connex-pp-heads-{ep.model}-{ep.stage_idx}-{ep.replica_idx}.json")
        self.heads = HeadState(path)
        self.stats = collections.Counter()
        ep.control_handlers.append(self._on_control)

    def _owner_silent_for(self) -> float:
        last = max(self._owner_seen, self.ep.last_step_from.get(self.owner, 0.0))
        return time.monotonic() - last

    def _on_control(self, msg: dict) -> None:
        kind, sender = msg.get("kind"), msg.get("from")
        if kind == HELLO:
            self.heads.remember(sender)
            if self.owner in (None, sender) or self._owner_silent_for() > self.takeover_s:
                if self.owner not in (None, sender):
                    log.warning("stage %s replica %s: %s takes over from silent owner %s", self.ep.stage_idx,
                                self.ep.replica_idx, sender, self.owner)
                    self.stats["takeovers"] += 1
                self.owner, self._owner_seen = sender, time.monotonic()
                self.ep.send_control(sender, {"kind": HELLO_OK, "owner": sender})
            else:
                self.stats["busy"] += 1
                self.ep.send_control(sender, {"kind": BUSY, "owner": self.owner})
        elif kind == PING:
            if sender == self.owner:
                self._owner_seen = time.monotonic()
            self.ep.send_control(sender, {"kind": PONG, "t": msg.get("t"), "done_seq": self.ep.done_seq,
                                          "next": self.ep.current_addr})
        elif kind == FAILOVER:
            self.ep.on_peer_dead(int(msg["target_stage"]), int(msg["target_replica"]),
                                 msg.get("reason", "stage 0 watchdog"))

    def announce(self) -> int:
        """Tell the stage-0 instances served before a restart that this replica
        is serving; returns how many were told."""
        for head in self.heads.heads:
            self.ep.send_control(head, {"kind": READY})
        return len(self.heads.heads)

    def dying(self, reason: str = "exiting") -> None:
        """Tell the owner (or every known head) to fail over now."""
        for head in [self.owner] if self.owner else self.heads.heads:
            self.ep.send_control(head, {"kind": DYING, "reason": reason})


@dataclass
class Hop:
    """What stage 0 knows of one replica on its route."""

    stage: int
    replica: int
    address: str
    pong: float = 0.0               # time of its last PONG
    done_seq: int = -1              # last step it answered, as of that PONG
    next: Optional[str] = None      # its downstream address, as of that PONG
    alive_since: float = 0.0        # its last HELLO_OK


def pick_stuck(route: Sequence[Hop], late: Sequence[int], t_ping: float) -> Tuple[Optional[Hop], str]:
    """The replica to fail over for the ``late`` steps after a PING sent at
    ``t_ping``: the first one on the route that did not answer; if all
    answered (a hung stream still answers), the first one that has not
    finished the oldest late step; else the last one.  (None, "") when no
    step is late any more."""
    if not late:
        return None, ""
    for hop in route:
        if hop.pong < t_ping:
            return hop, "step timeout, no pong"
    oldest = min(late)
    behind = next((h for h in route if h.done_seq < oldest), route[-1] if route else None)
    return behind, f"step {oldest:#x} timeout, stage answers but is stuck"


class ChainWatchdog:
    """Stage 0's side of the protocol: HELLO to every downstream it routes to,
    reacts to HELLO_OK / BUSY / READY / DYING, and finds hung stages.

    A hung replica further down than our own downstream is failed over by
    its upstream replica (FAILOVER) and reported through ``report``.

    Step timeout: the fixed ``step_timeout`` until ``min_samples`` steps came
    back; then ``factor`` x the slowest measured step at least as large as the
    late one (clamped to [``min_timeout``, ``step_timeout``]) -- after many
    small decode steps a long prefill is not a hang, and a step larger than
    any measured keeps the fixed backstop.  A late step triggers a PING of
    the whole route (each PONG names the next hop), then :func:`pick_stuck`."""

    def __init__(self, ep, link, step_timeout: float = 60.0, min_timeout: float = 2.0, factor: float = 20.0,
                 min_samples: int = 32, ping_wait_s: float = 1.0, period_s: float = 0.5,
                 report: Optional[Callable[[int, int, str], None]] = None):
        self.ep, self.link = ep, link
        self.step_timeout, self.min_timeout, self.factor = step_timeout, min_timeout, factor
        self.min_samples = min_samples
        self.ping_wait_s, self.period_s = ping_wait_s, period_s
        self.report = report           # (stage, replica, reason) -> tell the membership service
        self.hops: Dict[Tuple[int, int], Hop] = {}
        self.samples: Deque[Tuple[float, int]] = collections.deque(maxlen=512)
        self.events: List[dict] = []
        self.stats = collections.Counter()
        self._lock = threading.Lock()
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None
        ep.control_handlers.append(self._on_control)
        ep.route_listeners.append(self._on_route)
        ep.failure_veto = self.vetoes
        link.step_listeners.append(self.record)

    # --------------------------------------------------------------- timeout
    def record(self, seconds: float, size: int) -> None:
        self.samples.append((seconds, size))

    def current_step_timeout(self, size: int = 0) -> float:
        if len(self.samples) < self.min_samples:
            return self.step_timeout
        slowest = max((s for s, n in self.samples if n >= size), default=None)
        if slowest is None:
            return self.step_timeout
        return min(self.step_timeout, max(self.min_timeout, self.factor * slowest))

    # --------------------------------------------------------------- control
    def _hop(self, msg: dict) -> Hop:
        key = (int(msg.get("stage", -1)), int(msg.get("replica", -1)))
        hop = self.hops.get(key)
        if hop is None:
            hop = self.hops[key] = Hop(key[0], key[1], msg.get("from", ""))
        if msg.get("from"):
            hop.address = msg["from"]
        return hop

    def hello(self, address: str) -> None:
        self.ep.send_control(address, {"kind": HELLO})

    def _on_route(self, stage: int, replica: int, address: str) -> None:
        self.hops.setdefault((stage, replica), Hop(stage, replica, address)).address = address
        self.hello(address)

    def _on_control(self, msg: dict) -> None:
        kind = msg.get("kind")
        hop = self._hop(msg)
        now = time.monotonic()
        if kind == HELLO_OK:
            hop.alive_since = hop.pong = now
            self.ep.on_peer_alive(hop.stage, hop.replica)
        elif kind == PONG:
            hop.pong, hop.done_seq, hop.next = now, int(msg.get("done_seq", -1)), msg.get("next")
        elif kind == READY:
            self.stats["ready"] += 1
            self.ep.on_peer_alive(hop.stage, hop.replica)
            self.hello(hop.address)
        elif kind in (DYING, BUSY):
            why = f"stage exiting ({msg.get('reason', '')})" if kind == DYING else f"owned by {msg.get('owner')}"
            self.stats[kind.lower()] += 1
            self._fail(hop, why)

    def answers_ping(self, hop: Hop, timeout_s: float = 0.5) -> bool:
        t = time.monotonic()
        self.ep.send_control(hop.address, {"kind": PING, "t": t})
        while time.monotonic() - t < timeout_s:
            if hop.pong >= t:
                return True
            time.sleep(0.01)
        return False

    def vetoes(self, stage: int, replica: int) -> bool:
        """True when a failure report about (stage, replica) is about an
        earlier incarnation: the replica said HELLO_OK less than
        ``REJOIN_GRACE_S`` ago and still answers a PING."""
        hop = self.hops.get((stage, replica))
        if hop is None or time.monotonic() - hop.alive_since > REJOIN_GRACE_S:
            return False
        if self.answers_ping(hop):
            self.stats["false_failures"] += 1
            log.info("ignoring a failure report for stage %s replica %s: it answers", stage, replica)
            return True
        return False

    # ------------------------------------------------------------ detection
    def _route(self) -> List[Hop]:
        """The route as last reported by PONGs, starting at our downstream."""
        route, addr, seen = [], self.ep.current_addr, set()
        by_addr = {h.address: h for h in self.hops.values()}
        while addr and addr in by_addr and addr not in seen:
            seen.add(addr)
            route.append(by_addr[addr])
            addr = by_addr[addr].next
        return route

    def _ping_route(self) -> float:
        t = time.monotonic()
        msg = {"kind": PING, "t": t}
        pinged = set()
        deadline = t + self.ping_wait_s
        while time.monotonic() < deadline:
            for hop in self._route():                 # a PONG may reveal the next hop: ping it too
                if hop.address not in pinged:
                    pinged.add(hop.address)
                    self.ep.send_control(hop.address, msg)
            time.sleep(0.02)
        return t

    def _fail(self, hop: Hop, reason: str) -> None:
        log.warning("stage 0: failing over stage %s replica %s (%s)", hop.stage, hop.replica, reason)
        self.events.append({"t": time.time(), "stage": hop.stage, "replica": hop.replica, "reason": reason})
        hop.alive_since = 0.0
        if hop.stage == self.ep.stage_idx + 1:
            self.ep.on_peer_dead(hop.stage, hop.replica, reason)
            return
        upstream = next((h for h in self._route() if h.next == hop.address), None)
        if upstream is not None:
            self.ep.send_control(upstream.address, {"kind": FAILOVER, "target_stage": hop.stage,
                                                    "target_replica": hop.replica, "reason": reason})
        if self.report is not None:
            self.report(hop.stage, hop.replica, reason)

    def check_once(self) -> Optional[Hop]:
        """One watchdog round; returns the replica it failed over, if any."""
        now = time.monotonic()
        late = [corr for corr, sent, size in self.link.pending_steps() if now - sent > self.current_step_timeout(size)]
        if not late:
            return None
        self.stats["late_rounds"] += 1
        t_ping = self._ping_route()
        still = set(c for c, _, _ in self.link.pending_steps())
        victim, why = pick_stuck(self._route(), [c for c in late if c in still], t_ping)
        if victim is None:
            return None
        self._fail(victim, why)
        return victim

    def start(self) -> "ChainWatchdog":
        def loop():
            while not self._stop.wait(self.period_s):
                try:
                    self.check_once()
                except Exception:  # noqa: BLE001 - the watchdog must keep running
                    log.exception("watchdog round failed")
        self._thread = threading.Thread(target=loop, daemon=True, name="cx-pp-watchdog")
        self._thread.start()
        return self

    def stop(self) -> None:
        self._stop.set()
