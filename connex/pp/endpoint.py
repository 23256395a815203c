"""Pipeline stage endpoint: the engine-neutral core of elastic PP (reference
``connex/pp/endpoint.py:276-2526``, ``ConnexTEEndpoint``).

One :class:`PipelineEndpoint` per stage process.  Stage 0 drives steps
(``new_step_id`` / ``send_step`` / ``recv_step`` / ``abandon_step``); later
stages answer (``recv_forward`` / ``send_reply``); the last stage replies to
the stage-0 endpoint named in the step (``origin``).  ``send_tensor_dict`` /
``recv_tensor_dict`` are the K=1 form.  It implements the
:class:`connex.pp.hooks.StepTransport` protocol, so
:class:`connex.pp.link.Stage0Link` / :class:`StageWorker` drive it.

Every message is a ``CONNEXTE`` signal (:mod:`connex.pp.wire`) with a ``G2``
tail (layout of the tensors, ack endpoint, origin, pickled non-tensor
fields), and the tensors travel by one of three data planes:

* ``link`` -- an elastic two-rank NCCL group per peer pair
  (:class:`connex_b200.parallel.pplink.PairLinks`; gloo on CPU): the sender
  posts the sends right after the signal, the receiver posts the receives in
  signal order on the link's own stream (device activations over NVLink);
* ``engine`` -- a registered host send ring read one-sided by the receiver
  through the native transfer engine, released by a ``CXACK`` (ring reuse
  by ack, :class:`connex.pp.ring.RegionTable`);
* ``inline`` -- the bytes ride in the ZeroMQ message.

Rules kept from the reference: K steps in flight, each under its own
correlation id ``incarnation << 32 | seq``; later stages drop ids K or more
behind the newest of an incarnation and answer duplicates from a reply cache
of the last K replies; stage 0's receive timeout adapts (max(base, 3 x the
slowest step)); a peer reported dead (membership event, engine event, or a
timeout confirmed by a refused TCP connect) bumps the chain epoch, which
fails every step sent before it at once (``step_stale``) so the caller
re-sends them to the newly selected replica (sticky routing,
:func:`connex.pp.routing.select_peer`).
"""
from __future__ import annotations

import json
import logging
import os
import pickle
import queue
import random
import socket
import threading
import time
from collections import defaultdict
from typing import Any, Dict, List, Optional, Tuple

import zmq

from connex.pp import wire
from connex.pp.hooks import NULL_METRICS
from connex.pp.ring import RegionTable
from connex.pp.routing import select_peer
from connex.pp.steps import CorrFilter, ReplyCache, StepIds

log = logging.getLogger("connex.pp.endpoint")

DEFAULT_RECV_TIMEOUT_S = float(os.getenv("CONNEXTE_RECV_TIMEOUT_MS", "8000")) / 1000
# CONNEXTE_TRACE=/path/prefix: append "time stage event corr" lines to
# <prefix>.stage<N>.txt (send called / signal posted / arrived / receive done)
# to rebuild the cross-stage timeline of each step.  CONNEXTE_PROFILE=1: log
# mean milliseconds per phase every CONNEXTE_PROFILE_EVERY receives.
TRACE_PREFIX = os.getenv("CONNEXTE_TRACE", "")
PROFILE = os.getenv("CONNEXTE_PROFILE", "0") == "1"
PROFILE_EVERY = int(os.getenv("CONNEXTE_PROFILE_EVERY", "64"))
# CONNEX_RS_STATS_S=N: every N seconds log the native engine's counters with
# this process's open file descriptors and resident memory (leak checks).
RS_STATS_S = float(os.getenv("CONNEX_RS_STATS_S", "0") or 0)
PROBE_TIMEOUT_S = float(os.getenv("CONNEXTE_PROBE_TIMEOUT_S", "0.5") or "0.5")
ACK_TIMEOUT_S = float(os.getenv("CONNEXTE_GDR_ACK_TIMEOUT_S", "10.0"))


def probe_tcp(address: Optional[str], timeout_s: float = PROBE_TIMEOUT_S) -> Optional[bool]:
    """Is something listening at ``tcp://host:port``?  True / False, or None
    when unknown.  The kernel answers for a live but busy process; a dead one
    refuses at once."""
    if not address or not address.startswith("tcp://"):
        return None
    hp = address[len("tcp://"):].split("#", 1)[0]
    host, _, port = hp.rpartition(":")
    host = host.strip("[]")
    try:
        with socket.create_connection((host, int(port)), timeout=timeout_s):
            return True
    except ConnectionRefusedError:
        return False
    except OSError:
        return None


class _Tracer:
    def __init__(self, prefix: str, stage: int):
        self.f = open(f"{prefix}.stage{stage}.txt", "a", buffering=1 << 16) if prefix else None
        self.stage = stage
        self.lock = threading.Lock()

    def __call__(self, event: str, corr) -> None:
        if self.f is not None:
            with self.lock:
                self.f.write(f"{time.time():.6f} {self.stage} {event} {corr}\n")

    def close(self) -> None:
        if self.f is not None:
            self.f.close()


class _Profiler:
    """Per-phase wall time (ms), logged as means every ``every`` receives."""

    def __init__(self, enabled: bool, every: int, stage: int):
        self.enabled, self.every, self.stage = enabled, every, stage
        self.acc: Dict[str, float] = defaultdict(float)
        self.n = 0

    def add(self, phase: str, seconds: float) -> None:
        if self.enabled:
            self.acc[phase] += seconds * 1e3

    def tick(self) -> None:
        if not self.enabled:
            return
        self.n += 1
        if self.n % self.every == 0:
            log.info("stage %s phases (mean ms over %d): %s", self.stage, self.every,
                     {k: round(v / self.every, 3) for k, v in self.acc.items()})
            self.acc.clear()


def process_stats() -> dict:
    """Open file descriptors and resident set size (MiB) of this process."""
    try:
        fds = len(os.listdir("/proc/self/fd"))
    except OSError:
        fds = -1
    try:
        with open("/proc/self/statm") as f:
            rss_mb = int(f.read().split()[1]) * os.sysconf("SC_PAGE_SIZE") / (1 << 20)
    except (OSError, ValueError, IndexError):
        rss_mb = -1.0
    return {"fds": fds, "rss_mb": round(rss_mb, 1)}


CONTROL_MAGIC = b"CXCTL"     # liveness-protocol messages (JSON) share the endpoint's sockets
ENGINE_ADDRESS_PREFIX = "cx="  # a listed address "cx=<url>": the replica's transfer engine (peer events)


class ChainFailed(RuntimeError):
    """Raised by the K=1 receive when the downstream chain failed over."""


class _Msg:
    __slots__ = ("corr", "td", "origin", "sender", "ready")

    def __init__(self, corr, td, origin, sender, ready=None):
        self.corr, self.td, self.origin, self.sender, self.ready = corr, td, origin, sender, ready


class PipelineEndpoint:
    def __init__(self, model: str, stage_idx: int, num_stages: int, replica_idx: int = 0, *, membership=None,
                 host: str = "127.0.0.1", port: int = 0, data: str = "auto", links=None, engine=None,
                 ring_bytes: int = 64 << 20, k: Optional[int] = None, recv_timeout_s: Optional[float] = None,
                 device: str = "cpu", metrics=NULL_METRICS):
        self.model, self.stage_idx, self.num_stages, self.replica_idx = model, stage_idx, num_stages, replica_idx
        self.is_first, self.is_last = stage_idx == 0, stage_idx == num_stages - 1
        self.membership = membership
        self.device = device
        self.metrics = metrics
        self.k = max(1, k if k is not None else int(os.getenv("CONNEX_PP_INFLIGHT", "1") or 1))
        self.base_timeout_s = recv_timeout_s if recv_timeout_s is not None else DEFAULT_RECV_TIMEOUT_S
        self.incarnation = random.getrandbits(31) | 1
        self.name = f"{model}|{stage_idx}|0|{replica_idx}"
        self.link_id = f"{self.name}@{self.incarnation:x}"     # unique per process incarnation
        self.links = links
        self.engine = engine
        self.data = data if data != "auto" else ("link" if links is not None else "engine" if engine else "inline")
        # sockets (owned by the I/O thread after start)
        self.ctx = zmq.Context()
        self.router = self.ctx.socket(zmq.ROUTER)
        self.router.setsockopt(zmq.LINGER, 0)
        port = port or self.router.bind_to_random_port(f"tcp://{host}")
        if port and not self.router.getsockopt(zmq.LAST_ENDPOINT):
            self.router.bind(f"tcp://{host}:{port}")
        self.address = f"tcp://{host}:{port}#{self.link_id}"   # '#': link identity of this endpoint
        self._dealers: Dict[str, zmq.Socket] = {}
        self._outq: "queue.Queue" = queue.Queue()
        self._wake_addr = f"inproc://cx-wake-{id(self)}"
        self._wake_rx = self.ctx.socket(zmq.PAIR)
        self._wake_rx.bind(self._wake_addr)
        self._wake_tx = self.ctx.socket(zmq.PAIR)
        self._wake_tx.connect(self._wake_addr)
        self._wake_lock = threading.Lock()
        # step state
        self.ids = StepIds(wire.make_corr(self.incarnation, 0))
        self.filter = CorrFilter(window=self.k)
        self.replies = ReplyCache(self.k)
        self.inbox: "queue.Queue[_Msg]" = queue.Queue()
        self._done: Dict[int, _Msg] = {}
        self._outstanding: set = set()
        self._cv = threading.Condition()
        self.chain_epoch = 0
        self._sent_epoch: Dict[int, int] = {}
        self._sent_at: Dict[int, float] = {}
        self.slowest_step_s = 0.0
        self.current: Optional[int] = None            # downstream replica (sticky)
        self.current_addr: Optional[str] = None
        self.deregistered: set = set()
        self.suspect: set = set()                    # (stage, replica) that missed a lease, being probed
        self._probe_threads: List[threading.Thread] = []
        self.codec = wire.LayoutCodec()
        self.stats = defaultdict(int)
        self.trace = _Tracer(TRACE_PREFIX, stage_idx)
        self.prof = _Profiler(PROFILE, PROFILE_EVERY, stage_idx)
        self._ring = None
        if self.data == "engine":
            self._setup_ring(ring_bytes)
        self._stop = threading.Event()
        self._send_lock = threading.Lock()      # a signal and its link sends stay together, per process
        self.auto_warm = False
        self._warm_threads: List[threading.Thread] = []
        # liveness protocol (connex.pp.liveness) and the transport peer watch
        self.control_handlers: List[Any] = []        # called with each control message (I/O thread)
        self.route_listeners: List[Any] = []         # called with (stage, replica, address) on a new downstream
        self.failure_veto = None                      # (stage, replica) -> True: ignore a failure report
        self.last_step_from: Dict[str, float] = {}    # stage-0 address -> time of its last step here
        self.done_seq = -1                            # the last step this stage answered
        self._watch_pump = None
        self._watch_engine = None
        self._watched: dict = {}            # (stage, replica) -> engine URL connected for peer events
        self._transport_up: set = set()
        self.last_transport_failover: Optional[dict] = None
        if membership is not None:
            self.attach_membership(membership)
        self._io = threading.Thread(target=self._io_loop, name=f"cx-pp-io-{stage_idx}", daemon=True)
        self._io.start()

    # ------------------------------------------------------------ plumbing
    @property
    def inflight(self) -> int:
        return self.k

    def _setup_ring(self, nbytes: int) -> None:
        import torch
        self._ring_t = torch.empty(nbytes, dtype=torch.uint8, pin_memory=torch.cuda.is_available())
        rc = self.engine.register_memory(self._ring_t.data_ptr(), nbytes)
        if rc != 0:
            raise RuntimeError(f"register_memory failed: {rc}")
        self._ring = RegionTable(nbytes)
        self._ring_lock = threading.Lock()
        # one-sided reads land in registered memory only: a receive buffer
        self._rx_t = torch.empty(nbytes, dtype=torch.uint8, pin_memory=torch.cuda.is_available())
        if self.engine.register_memory(self._rx_t.data_ptr(), nbytes) != 0:
            raise RuntimeError("register_memory (receive buffer) failed")

    def _post(self, address: str, frames: List[bytes]) -> None:
        self._outq.put((address, frames))
        with self._wake_lock:
            self._wake_tx.send(b"x")

    def _dealer(self, address: str) -> zmq.Socket:
        s = self._dealers.get(address)
        if s is None:
            s = self.ctx.socket(zmq.DEALER)
            s.setsockopt(zmq.LINGER, 0)
            s.setsockopt(zmq.IDENTITY, f"{self.name}-{os.urandom(4).hex()}".encode())
            s.setsockopt(zmq.SNDHWM, 10000)
            s.connect(address.split("#", 1)[0])
            self._dealers[address] = s
        return s

    def _io_loop(self) -> None:
        poller = zmq.Poller()
        poller.register(self.router, zmq.POLLIN)
        poller.register(self._wake_rx, zmq.POLLIN)
        next_stats = time.monotonic() + RS_STATS_S
        while not self._stop.is_set():
            try:
                ready = dict(poller.poll(50))
            except zmq.ZMQError:
                break
            if RS_STATS_S > 0 and time.monotonic() >= next_stats:
                next_stats = time.monotonic() + RS_STATS_S
                eng = self.engine.stats() if self.engine is not None and hasattr(self.engine, "stats") else {}
                log.info("stage %s engine %s process %s", self.stage_idx, eng, process_stats())
            if self._wake_rx in ready:
                while True:
                    try:
                        self._wake_rx.recv(zmq.NOBLOCK)
                    except zmq.Again:
                        break
            while True:
                try:
                    addr, frames = self._outq.get_nowait()
                except queue.Empty:
                    break
                try:
                    self._dealer(addr).send_multipart(frames, copy=False)
                except zmq.ZMQError as e:
                    log.warning("stage %s: send to %s failed: %s", self.stage_idx, addr, e)
            if self.router in ready:
                while True:
                    try:
                        frames = self.router.recv_multipart(zmq.NOBLOCK)
                    except zmq.Again:
                        break
                    try:
                        self._on_message(frames[1:])
                    except Exception:  # noqa: BLE001 - one bad message must not stop the loop
                        log.exception("stage %s: bad message", self.stage_idx)

    # ------------------------------------------------------------- packing
    def _pack(self, td: dict):
        import torch
        tensors = [(k, v) for k, v in td.items() if isinstance(v, torch.Tensor)]
        nt = {k: v for k, v in td.items() if not isinstance(v, torch.Tensor)}
        key = tuple((k, str(v.dtype).replace("torch.", ""), tuple(v.shape)) for k, v in tensors)
        layout, total, layout_b = self.codec.layout_for(key, [v.numel() * v.element_size() for _, v in tensors])
        return tensors, nt, layout, total, layout_b

    def _send(self, address: str, td: dict, corr: int, origin: str) -> None:
        import torch
        self.trace("send_called", corr)
        t0 = time.perf_counter()
        tensors, nt, layout, total, layout_b = self._pack(td)
        nt_b = pickle.dumps(nt) if nt else b""
        token, src, extra = 0, 0, []
        if self.data == "engine" and tensors:
            now = time.monotonic()
            with self._ring_lock:
                for old in self._ring.collect(now):      # temp buffers whose reader is done
                    self.engine.unregister_memory(old.data_ptr())
                got = self._ring.alloc(total, now, ACK_TIMEOUT_S, True)
                if got is not None:
                    start, token = got
                    buf = self._ring_t[start:start + total]
                else:       # ring busy: a registered temporary buffer, freed on its ack
                    buf = torch.empty(total, dtype=torch.uint8, pin_memory=torch.cuda.is_available())
                    if self.engine.register_memory(buf.data_ptr(), total) != 0:
                        raise RuntimeError("cannot register a temporary send buffer")
                    token = self._ring.add_temp(buf, now, ACK_TIMEOUT_S, True)
                    self.stats["ring_full"] += 1
            for (_, _, _, off, nb), (_, v) in zip(layout, tensors):
                buf[off:off + nb].copy_(v.detach().contiguous().view(-1).view(torch.uint8))
            src = buf.data_ptr()
        elif self.data == "inline" and tensors:
            buf = bytearray(total)
            for (_, _, _, off, nb), (_, v) in zip(layout, tensors):
                buf[off:off + nb] = v.detach().contiguous().view(-1).view(torch.uint8).cpu().numpy().tobytes()
            extra = [bytes(buf)]
        url = (self.engine.local_url if self.data == "engine" else self.link_id).encode()
        tail = wire.encode_g2(token, layout_b or b"", self.address.encode(), origin.encode(), nt_b)
        with self._send_lock:
            self._post(address, [wire.encode_signal(src, total, url, corr, tail)] + extra)
            if self.data == "link" and tensors:
                self.links.open_tx(self._peer_name(address)).send([v.contiguous() for _, v in tensors])
        self.stats["sent"] += 1
        self.trace("signaled", corr)
        self.prof.add("send", time.perf_counter() - t0)

    def send_control(self, address: str, msg: dict) -> None:
        """A liveness-protocol message (:mod:`connex.pp.liveness`) to the
        endpoint at ``address``; it carries this endpoint's identity."""
        body = dict(msg, **{"from": self.address, "stage": self.stage_idx, "replica": self.replica_idx})
        self._post(address, [CONTROL_MAGIC + json.dumps(body).encode()])

    def _on_control(self, body: bytes) -> None:
        msg = json.loads(body[len(CONTROL_MAGIC):])
        self.stats["control_" + str(msg.get("kind", "?")).lower()] += 1
        for handler in list(self.control_handlers):
            handler(msg)

    def _peer_name(self, address: str) -> str:
        """Link identity of the endpoint at ``address`` (carried after '#')."""
        return address.split("#", 1)[1] if "#" in address else address

    def _on_message(self, frames: List[bytes]) -> None:
        body = frames[0]
        if body.startswith(CONTROL_MAGIC):
            self._on_control(body)
            return
        tok = wire.decode_ack(body)
        if tok is not None:
            if self._ring is not None:
                with self._ring_lock:
                    self._ring.ack(tok)
            return
        sig = wire.decode_signal(body)
        if sig.tag != wire.TAG_G2:
            raise ValueError("unsupported signal tail")
        token, layout_b, ack_ep, origin, nt_b = wire.decode_g2(sig.tail[2:])
        layout = self.codec.parse(layout_b) if layout_b else []
        td: Dict[str, Any] = pickle.loads(nt_b) if nt_b else {}
        ready = None
        if layout:
            ready = self._receive_tensors(sig, layout, td, frames[1:])
        if token and ack_ep:
            self._post(ack_ep, [wire.encode_ack(token)])
        self.trace("arrived", sig.corr)
        self._deliver(_Msg(sig.corr, td, origin, sig.url, ready))

    def _receive_tensors(self, sig, layout, td, extra):
        import torch
        dts = {n: getattr(torch, n) for n in wire.DT_NAMES if hasattr(torch, n)}
        if self.data == "link":
            link = self.links.open_rx(sig.url)
            out = {k: torch.empty(shape, dtype=dts[dt], device=self.device) for k, dt, shape, _, _ in layout}
            link.recv(list(out.values()))
            td.update(out)
            return link.done_event()
        if self.data == "engine":
            if sig.total <= self._rx_t.numel():
                data, tmp = self._rx_t[:sig.total], None
            else:
                data = tmp = torch.empty(sig.total, dtype=torch.uint8)
                self.engine.register_memory(tmp.data_ptr(), sig.total)
            try:
                rc = self.engine.transfer_sync_read(sig.url, data.data_ptr(), sig.src_ptr, sig.total)
            finally:
                if tmp is not None:
                    self.engine.unregister_memory(tmp.data_ptr())
            if rc != 0:
                raise RuntimeError(f"one-sided read from {sig.url} failed: {rc}")
        else:
            data = torch.frombuffer(bytearray(extra[0]), dtype=torch.uint8)
        for k, dt, shape, off, nb in layout:
            t = data[off:off + nb].view(dts[dt]).view(shape).clone()
            td[k] = t.to(self.device) if self.device != "cpu" else t
        return None

    def _deliver(self, m: _Msg) -> None:
        if self.is_first:
            with self._cv:
                if m.corr in self._outstanding:
                    self._done[m.corr] = m
                    self._cv.notify_all()
                else:
                    self.stats["late_replies"] += 1
            return
        self.last_step_from[m.origin] = time.monotonic()
        cached = self.replies.get(m.corr)
        if cached is not None:          # duplicate of an answered step: answer again
            self.stats["dedup_replies"] += 1
            self._send_reply_now(cached[0], m.corr, cached[1])
            return
        if not self.filter.accept(m.corr):
            self.stats["stale_dropped"] += 1
            return
        self.inbox.put(m)

    # ------------------------------------------------------------- routing
    def _downstream(self) -> Optional[str]:
        if self.membership is None:
            return self.current_addr
        peers = self.membership.get_pipeline_peers()
        addr, rep, new = select_peer(peers, self.stage_idx + 1, self.stage_idx, self.replica_idx, self.current,
                                     self.deregistered)
        if addr is not None and (new or rep != self.current):
            if self.current is not None and rep != self.current:
                self.chain_epoch += 1
            self.current, self.current_addr = rep, addr
            self._announce_route()
        return addr

    def _announce_route(self) -> None:
        for listener in list(self.route_listeners):
            try:
                listener(self.stage_idx + 1, self.current, self.current_addr)
            except Exception:  # noqa: BLE001
                log.exception("route listener")

    def set_downstream(self, address: str, replica_idx: int = 0) -> None:
        """Fixed downstream (no membership)."""
        if self.current_addr is not None and address != self.current_addr:
            self.chain_epoch += 1
        changed = address != self.current_addr
        self.current, self.current_addr = replica_idx, address
        if changed:
            self._announce_route()

    def on_peer_dead(self, stage_idx: int, replica_idx: int, reason: str = "") -> bool:
        """A peer is gone; True if it was this endpoint's downstream."""
        self.suspect.discard((stage_idx, replica_idx))
        self.deregistered.add((stage_idx, replica_idx))
        if self.links is not None and self.membership is not None:
            for r in self.membership.get_stage_peers(stage_idx):
                if r.lid.replica_idx == replica_idx and r.addresses:
                    self.links.drop_peer(self._peer_name(r.addresses[0]))
        if stage_idx == self.stage_idx + 1 and replica_idx == self.current:
            log.warning("stage %s: downstream replica %s dead (%s); failing over", self.stage_idx, replica_idx,
                        reason)
            self.current, self.current_addr = None, None
            self.chain_epoch += 1
            with self._cv:
                self._cv.notify_all()
            self.stats["failovers"] += 1
            return True
        return False

    def on_peer_alive(self, stage_idx: int, replica_idx: int) -> None:
        self.deregistered.discard((stage_idx, replica_idx))

    # ---------------------------------------------------- transport watch
    def watch_peers(self, engine, urls: Optional[Dict[Tuple[int, int], str]] = None) -> None:
        """First tier of failure detection: follow ``engine``'s peer events
        (the native engine reports a peer's socket reset or heartbeat loss
        within milliseconds).  ``urls``: (stage, replica) -> engine URL of
        downstream replicas to connect to (more with :meth:`watch_peer`).

        A ``failed`` event about a downstream replica whose link was up
        fails it over at once -- unless :attr:`failure_veto` says the report
        is about an earlier incarnation; a failure by heartbeat timeout only
        makes it suspect (the TCP probe decides)."""
        from connex.pd.group import EventPump
        self._watch_engine = engine
        for (stage, replica), url in (urls or {}).items():
            self.watch_peer(stage, replica, url)
        if self.membership is not None:
            for r in self.membership.get_stage_peers(self.stage_idx + 1):
                self._watch_listed(r.lid.stage_idx, r.lid.replica_idx, r.addresses)
        self._watch_pump = EventPump(engine, self._on_transport_event, name=f"cx-pp-watch-{self.stage_idx}").start()

    def watch_peer(self, stage_idx: int, replica_idx: int, url: str) -> bool:
        """Connect the watch engine to a downstream replica's engine (once per
        incarnation: a failed peer is connected again when it is listed again)."""
        if self._watch_engine is None or self._watched.get((stage_idx, replica_idx)) == url:
            return False
        self._watched[(stage_idx, replica_idx)] = url
        try:
            return bool(self._watch_engine.connect(url))
        except Exception as e:  # noqa: BLE001 - the lease tier still covers this peer
            log.warning("stage %s: cannot watch %s: %s", self.stage_idx, url, e)
            return False

    def _watch_listed(self, stage_idx: int, replica_idx: int, addresses) -> None:
        """Watch a listed downstream replica that advertises an engine
        (an address ``cx=<engine url>`` beside its step address)."""
        if stage_idx != self.stage_idx + 1:
            return
        for a in addresses or ():
            if isinstance(a, str) and a.startswith(ENGINE_ADDRESS_PREFIX):
                self.watch_peer(stage_idx, replica_idx, a[len(ENGINE_ADDRESS_PREFIX):])

    def _on_transport_event(self, ev: dict) -> None:
        from connex.pd.group import is_timeout, peer_key
        key = peer_key(ev)
        if key is None or key[0] != self.model or key[1] != self.stage_idx + 1:
            return
        peer = (key[1], key[3])
        if ev.get("type") in ("up", "joined"):
            self._transport_up.add(peer)
            return
        if ev.get("type") != "failed" or peer not in self._transport_up:
            return
        self._transport_up.discard(peer)
        self._watched.pop(peer, None)
        t_event = time.monotonic()
        if is_timeout(ev):
            self.stats["transport_suspects"] += 1
            if peer == (self.stage_idx + 1, self.current) and self.current_addr is not None:
                alive = probe_tcp(self.current_addr)
                if alive is False:
                    self.on_peer_dead(peer[0], peer[1], "heartbeat lost, probe refused")
            return
        if self.failure_veto is not None and self.failure_veto(*peer):
            return
        self.stats["transport_failovers"] += 1
        self.on_peer_dead(peer[0], peer[1], f"transport: {ev.get('reason', 'failed')}")
        self.last_transport_failover = {"peer": peer, "event_t": t_event, "failover_t": time.monotonic(),
                                        "reason": ev.get("reason")}

    def attach_membership(self, membership) -> None:
        """Route with ``membership`` and follow its deregister / register events."""
        self.membership = membership
        if hasattr(membership, "on_event"):
            from connex.front_router import EventType
            membership.on_event(EventType.ENDPOINT_DEREGISTERED, self._on_membership_event)
            membership.on_event(EventType.ENDPOINT_UNHEALTHY, self._on_membership_unhealthy)
            membership.on_event(EventType.ENDPOINT_REGISTERED, self._on_membership_join)

    def _on_membership_event(self, ev) -> None:
        payload = getattr(ev, "payload", {}) or {}
        lid = payload.get("lid") or {}
        if "stage_idx" in lid:
            self.on_peer_dead(lid["stage_idx"], lid.get("replica_idx", 0), payload.get("reason", "event"))

    def _on_membership_unhealthy(self, ev) -> None:
        """A missed lease makes a peer *suspect*, not dead: only our own
        downstream matters, and it is probed in the background.  A refused
        connect confirms the death and fails over now (before the lease's
        grace ends); a peer that still accepts connects is kept (a busy
        process can miss a heartbeat)."""
        payload = getattr(ev, "payload", {}) or {}
        lid = payload.get("lid") or {}
        if "stage_idx" not in lid:
            return
        key = (lid["stage_idx"], lid.get("replica_idx", 0))
        if key != (self.stage_idx + 1, self.current):
            return
        self.suspect.add(key)
        addr = self.current_addr

        def probe():
            alive = probe_tcp(addr)
            if alive is False and key in self.suspect:
                self.on_peer_dead(key[0], key[1], "unhealthy, probe refused")
            else:
                self.stats["suspect_alive"] += 1
        t = threading.Thread(target=probe, daemon=True, name="cx-pp-probe")
        t.start()
        self._probe_threads.append(t)

    def _on_membership_join(self, ev) -> None:
        payload = getattr(ev, "payload", {}) or {}
        lid = payload.get("lid") or {}
        if "stage_idx" in lid:
            self.suspect.discard((lid["stage_idx"], lid.get("replica_idx", 0)))
            self.on_peer_alive(lid["stage_idx"], lid.get("replica_idx", 0))
            addrs = payload.get("addresses") or []
            if self._watch_engine is not None:
                self._watch_listed(lid["stage_idx"], lid.get("replica_idx", 0), addrs)
            if self.auto_warm and self.is_first and lid["stage_idx"] == 1 and addrs:
                t = threading.Thread(target=self.warm, args=(addrs[0],), daemon=True, name="cx-pp-warm")
                t.start()
                self._warm_threads.append(t)

    # ------------------------------------------------------------- warm-up
    def warm(self, address: str, timeout_s: float = 120.0) -> bool:
        """Send one empty ``warmup`` step through the chain starting at
        ``address`` and wait for it to come back (stage 0), so the data-plane
        links of a (new) replica are set up before traffic is routed to it."""
        import torch
        corr = self.new_step_id()
        w = torch.zeros(8, dtype=torch.bfloat16, device=self.device)
        try:
            self.send_step({"kind": "warmup", "w": w}, corr, dst=address)
            return self.recv_step(corr, timeout_s) is not None
        finally:
            self.abandon_step(corr)

    def warm_stage(self, stage_idx: int = 1) -> int:
        """Warm every listed replica of ``stage_idx``; returns how many answered."""
        if self.membership is None:
            return 0
        return sum(self.warm(r.addresses[0]) for r in self.membership.get_stage_peers(stage_idx) if r.addresses)

    def confirm_peer_failure(self) -> bool:
        """After a timeout: probe the downstream; a refused connect confirms death."""
        alive = probe_tcp(self.current_addr)
        if alive is False and self.current is not None:
            return self.on_peer_dead(self.stage_idx + 1, self.current, "probe refused")
        return False

    def downstream_healthy(self) -> bool:
        addr = self._downstream()
        return addr is not None and (self.stage_idx + 1, self.current) not in self.deregistered

    def step_stale(self, corr: int) -> bool:
        e = self._sent_epoch.get(corr)
        return e is not None and e != self.chain_epoch

    def _recv_timeout_s(self) -> float:
        return max(self.base_timeout_s, 3.0 * self.slowest_step_s)

    # --------------------------------------------------------- stage-0 API
    def new_step_id(self) -> int:
        with self._cv:                   # several threads may start steps (K > 1)
            c = self.ids.next()
            self._outstanding.add(c)
        return c

    def send_step(self, td: dict, corr: int, dst: Optional[str] = None) -> None:
        addr = dst or self._downstream()
        if addr is None:
            raise ConnectionError(f"stage {self.stage_idx}: no downstream replica")
        self._sent_epoch[corr] = self.chain_epoch
        self._sent_at.setdefault(corr, time.monotonic())
        self._send(addr, td, corr, self.address)

    def recv_step(self, corr: int, timeout_s: Optional[float] = None) -> Optional[dict]:
        w0 = time.perf_counter()
        deadline = time.monotonic() + (self._recv_timeout_s() if timeout_s is None else timeout_s)
        with self._cv:
            while corr not in self._done:
                if self.step_stale(corr):
                    return None
                left = deadline - time.monotonic()
                if left <= 0:
                    break
                self._cv.wait(min(left, 0.05))
            m = self._done.pop(corr, None)
            if m is not None:
                self._outstanding.discard(corr)
        if m is None:
            self.confirm_peer_failure()
            return None
        if m.ready is not None:
            import torch
            torch.cuda.current_stream().wait_event(m.ready)
        t0 = self._sent_at.pop(corr, None)
        if t0 is not None:
            dt = time.monotonic() - t0
            self.slowest_step_s = max(self.slowest_step_s * 0.99, dt)
            self.metrics.observe("step_latency", dt)
        self._sent_epoch.pop(corr, None)
        self.trace("recv_done", corr)
        self.prof.add("recv_wait", time.perf_counter() - w0)
        self.prof.tick()
        return m.td

    def abandon_step(self, corr: int) -> None:
        with self._cv:
            self._outstanding.discard(corr)
            self._done.pop(corr, None)
        self._sent_epoch.pop(corr, None)
        self._sent_at.pop(corr, None)

    # ------------------------------------------------------ later stages
    def recv_forward(self, timeout_s: Optional[float] = None):
        w0 = time.perf_counter()
        try:
            m = self.inbox.get(timeout=self._recv_timeout_s() if timeout_s is None else timeout_s)
        except queue.Empty:
            return None, None
        self.trace("recv_done", m.corr)
        self.prof.add("recv_wait", time.perf_counter() - w0)
        self.prof.tick()
        if m.ready is not None:
            import torch
            torch.cuda.current_stream().wait_event(m.ready)
        return m.td, (m.corr, m.origin)

    def send_reply(self, td: dict, ctx: Tuple[int, str]) -> None:
        corr, origin = ctx
        self.done_seq = corr
        self.replies.put(corr, (td, origin))
        self._send_reply_now(td, corr, origin)

    def _send_reply_now(self, td: dict, corr: int, origin: str) -> None:
        addr = origin if self.is_last else self._downstream()
        if addr is None:
            raise ConnectionError(f"stage {self.stage_idx}: nowhere to send step {corr:#x}")
        self._send(addr, td, corr, origin)

    # ------------------------------------------------------------ K = 1 API
    def send_tensor_dict(self, td: dict) -> None:
        if self.is_first:
            self._k1 = self.new_step_id()
            self.send_step(td, self._k1)
        else:
            self.send_reply(td, self._k1_ctx)

    def recv_tensor_dict(self, timeout_s: Optional[float] = None) -> Optional[dict]:
        if self.is_first:
            td = self.recv_step(self._k1, timeout_s)
            if td is None and self.step_stale(self._k1):
                raise ChainFailed(f"stage 0: chain failed over during step {self._k1:#x}")
            return td
        td, self._k1_ctx = self.recv_forward(timeout_s)
        return td

    def close(self) -> None:
        self._stop.set()
        if self._watch_pump is not None:
            self._watch_pump.stop()
        self._io.join(timeout=2)
        self.trace.close()
        for s in list(self._dealers.values()) + [self.router, self._wake_rx, self._wake_tx]:
            s.close(0)
        if self._ring is not None:
            self.engine.unregister_memory(self._ring_t.data_ptr())
            self.engine.unregister_memory(self._rx_t.data_ptr())
        self.ctx.term()


ConnexTEEndpoint = PipelineEndpoint
