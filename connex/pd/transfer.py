"""Pull-based KV block transfer between a prefill and a decode instance.

Prefill side -- :class:`KVProducer`
    After a request's prefill the engine *holds* its KV blocks under a
    transfer id.  Holds live in a :class:`LeaseTable`: every ``acquire``
    renews a hold's lease, a hold nobody acquires for ``retain_s`` expires,
    and a ``release`` frees it (after all ``of`` readers of a multi-reader
    TP pull released; a single-reader release from anyone but the last
    acquirer is ignored as stale -- a replacement decode instance may be
    re-pulling).  A release that arrives before its hold leaves a tombstone
    so the late hold is freed at once.  Freed and expired requests are handed
    back to the engine by :meth:`KVProducer.take_finished`.

    The control channel is a ZeroMQ ROUTER speaking msgpack ``{"op": ...}``:
    ``meta`` (incarnation, data-plane URL / backend, engine id, block size,
    device, KV layouts), ``acquire`` (the held block ids), ``release``,
    ``ping``.  A reply that refers to a host-staging copy still in flight is
    sent only once that copy has completed.

Decode side -- :class:`KVConsumer`
    A pull is a :class:`_PullJob`: acquire (retrying while the producer does
    not know the transfer yet), pick the remote blocks, fetch the producer's
    meta (cached per address, refreshed when the producer's incarnation
    changes), plan the fewest one-sided reads (whole blocks, or a head range
    for a heterogeneous-TP source), check that every destination lies in the
    registered KV memory, read, optionally release.  Results come back from
    :meth:`KVConsumer.take_done` as :class:`PullResult` objects -- a failed
    pull is reported, never raised.

Keeping a hold until it is released (not freeing it after the first read)
lets a replacement decode instance re-pull the prompt's KV after a decode
death instead of re-running the prefill.  Wire parity:
``connex/pd/transfer.py:148-195`` of the reference (op names, fields and
reply keys); the decomposition here is this module's own.
"""
from __future__ import annotations

import logging
import os
import threading
import time
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Sequence, Set, Tuple

import msgpack
import zmq

from connex.pd.host_staging import block_ranges, register_with_staging
from connex.pd.kv_layout import TPSource, TensorLayout, head_read_ops, read_ops, register_spans

log = logging.getLogger("connex.pd")
PROTO_VERSION = 1
_TOMBSTONE_CAP = 100_000


def _pack(o) -> bytes:
    return msgpack.packb(o, use_bin_type=True)


def _unpack(b: bytes):
    return msgpack.unpackb(b, raw=False)


# =========================================================== prefill side
@dataclass
class Lease:
    """One held transfer."""

    req_id: str
    blocks: List[int]
    expires: float
    staged: Any = None                    # host-staging completion event, if any
    acquires: int = 0
    owner: Optional[str] = None           # last acquirer
    releasers: Set[str] = field(default_factory=set)


class LeaseTable:
    """Held transfers by transfer id, with lease expiry and release rules."""

    def __init__(self, retain_s: float, clock=time.monotonic):
        self.retain_s = retain_s
        self.clock = clock
        self.leases: Dict[str, Lease] = {}
        self.tombstones: Set[str] = set()       # released before their hold arrived
        self.freed: Set[str] = set()            # request ids the engine may free
        self.counts = {"holds": 0, "acquires": 0, "releases": 0, "expired": 0, "unknown": 0}

    def hold(self, tid: str, req_id: str, blocks: Sequence[int], staged=None) -> bool:
        """False (and the request is freed at once) when already released."""
        if tid in self.tombstones:
            self.tombstones.discard(tid)
            self.freed.add(req_id)
            return False
        self.leases[tid] = Lease(req_id, list(blocks), self.clock() + self.retain_s, staged)
        self.counts["holds"] += 1
        return True

    def acquire(self, tid: str, who: Optional[str]) -> Optional[Lease]:
        lease = self.leases.get(tid)
        if lease is None:
            self.counts["unknown"] += 1
            return None
        lease.acquires += 1
        lease.owner = who or lease.owner
        lease.expires = self.clock() + self.retain_s
        self.counts["acquires"] += 1
        return lease

    def release(self, tid: str, who: Optional[str], of: int) -> dict:
        self.counts["releases"] += 1
        lease = self.leases.get(tid)
        if lease is None:
            if len(self.tombstones) >= _TOMBSTONE_CAP:
                self.tombstones.clear()
            self.tombstones.add(tid)
            return {"ok": True}
        if of <= 1:
            if who and lease.owner and who != lease.owner:
                self.counts["stale_releases"] = self.counts.get("stale_releases", 0) + 1
                return {"ok": True, "stale": True}
        else:
            lease.releasers.add(who)
            if len(lease.releasers) < of:
                return {"ok": True, "pending": of - len(lease.releasers)}
        self._free(tid)
        return {"ok": True}

    def _free(self, tid: str) -> None:
        self.freed.add(self.leases.pop(tid).req_id)

    def drop(self, tid: str) -> None:
        self.leases.pop(tid, None)

    def expire(self) -> None:
        now = self.clock()
        for tid in [t for t, l in self.leases.items() if l.expires < now]:
            self._free(tid)
            self.counts["expired"] += 1

    def take_freed(self) -> Set[str]:
        out, self.freed = self.freed, set()
        return out


def _event_done(ev) -> bool:
    try:
        return bool(ev.query())
    except Exception:  # noqa: BLE001 - an event without query(): wait for it
        ev.synchronize()
        return True


class _ControlServer:
    """ROUTER loop: ``answer(msg) -> (reply, wait_event)``; replies whose
    event has not completed are held back and sent once it has."""

    def __init__(self, answer, bind_ip: str, port: int):
        self._answer = answer
        self.sock = zmq.Context.instance().socket(zmq.ROUTER)
        self.sock.setsockopt(zmq.LINGER, 0)
        if port:
            self.sock.bind(f"tcp://{bind_ip}:{port}")
            self.port = port
        else:
            self.port = self.sock.bind_to_random_port(f"tcp://{bind_ip}")
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._loop, name="connex-pd-producer", daemon=True)
        self._thread.start()

    def _loop(self) -> None:
        deferred: List[Tuple[Any, list, dict]] = []
        while not self._stop.is_set():
            if self.sock.poll(1 if deferred else 100):
                *route, body = self.sock.recv_multipart()
                try:
                    reply, ev = self._answer(_unpack(body))
                except Exception as e:  # noqa: BLE001 - a bad request gets an error reply
                    reply, ev = {"ok": False, "why": f"error: {e}"}, None
                deferred.append((ev, route, reply))
            keep = []
            for ev, route, reply in deferred:
                if ev is None or _event_done(ev):
                    self.sock.send_multipart(route + [_pack(reply)])
                else:
                    keep.append((ev, route, reply))
            deferred = keep

    def close(self) -> None:
        self._stop.set()
        self._thread.join(timeout=2)
        self.sock.close(0)


class KVProducer:
    def __init__(self, plane, layouts: Sequence[TensorLayout], bind_ip: str = "0.0.0.0", port: int = 0,
                 retain_s: float = 60.0, engine_id: str = "", block_size: int = 0, register: bool = True,
                 device: str = ""):
        self.plane = plane
        self.layouts = list(layouts)
        self.retain_s = retain_s
        self.engine_id = engine_id
        self.inc = os.urandom(8).hex()
        self.block_size = block_size
        self.device = device
        self.table = LeaseTable(retain_s)
        self._lock = threading.Lock()
        self._staging = register_with_staging(plane, register_spans(self.layouts), "KV producer") if register \
            else getattr(plane, "_connex_staging", None)
        self._server = _ControlServer(self._answer, bind_ip, port)
        self.port = self._server.port

    @property
    def stats(self) -> dict:
        return self.table.counts

    # ----------------------------------------------------------- engine side
    def hold(self, req_id: str, transfer_id: str, blocks: Sequence[int]) -> None:
        with self._lock:
            if transfer_id in self.table.tombstones:
                self.table.hold(transfer_id, req_id, blocks)       # frees it at once
                return
        staged = None
        if self._staging is not None:
            staged = self._staging.stage_out(block_ranges(self.layouts, blocks))
        with self._lock:
            self.table.hold(transfer_id, req_id, blocks, staged)

    def drop(self, transfer_id: str) -> None:
        with self._lock:
            self.table.drop(transfer_id)

    def take_finished(self) -> set:
        """Request ids whose blocks the engine may free now (released or expired)."""
        with self._lock:
            self.table.expire()
            return self.table.take_freed()

    def held(self) -> int:
        with self._lock:
            return len(self.table.leases)

    # ---------------------------------------------------------- control side
    def meta(self) -> dict:
        layouts = [self._staging.translate(lo) if self._staging else lo for lo in self.layouts]
        d = {"ok": True, "v": PROTO_VERSION, "inc": self.inc, "url": self.plane.local_url,
             "backend": self.plane.name, "engine_id": self.engine_id, "block_size": self.block_size,
             "device": self.device, "layouts": [lo.to_dict() for lo in layouts]}
        describe = getattr(self.plane, "describe", None)
        if describe is not None and self._staging is None:
            d["spans"] = describe()
        return d

    def _answer(self, m: dict):
        op = m.get("op")
        if op == "meta":
            return self.meta(), None
        with self._lock:
            if op == "acquire":
                lease = self.table.acquire(m.get("tid"), m.get("who"))
                if lease is None:
                    return {"ok": False, "why": "unknown"}, None
                return {"ok": True, "blocks": lease.blocks, "inc": self.inc}, lease.staged
            if op == "release":
                return self.table.release(m.get("tid"), m.get("who"), int(m.get("of") or 1)), None
            if op == "ping":
                return {"ok": True, "held": len(self.table.leases)}, None
        return {"ok": False, "why": f"bad op {op!r}"}, None

    def answer(self, m: dict) -> dict:
        """Handle one control message in-process (no staging wait)."""
        return self._answer(m)[0]

    def close(self) -> None:
        self._server.close()


# ============================================================ decode side
@dataclass
class PullResult:
    req_id: str
    ok: bool
    why: str = ""
    nbytes: int = 0
    seconds: float = 0.0
    failed_blocks: List[int] = field(default_factory=list)


class _PeerMeta:
    """A producer's ``meta`` reply."""

    def __init__(self, d: dict):
        self.url = d["url"]
        self.backend = d.get("backend")
        self.engine_id = d.get("engine_id")
        self.inc = d.get("inc")
        self.block_size = d.get("block_size", 0)
        self.device = d.get("device", "")
        self.layouts = [TensorLayout.from_dict(x) for x in d["layouts"]]
        self.spans = d.get("spans")


class _ControlPool:
    """REQ sockets per producer address, reused between calls; a socket that
    timed out or failed is closed (a REQ socket cannot be reused then)."""

    def __init__(self, timeout_ms: int):
        self.timeout_ms = timeout_ms
        self._ctx = zmq.Context.instance()
        self._idle: Dict[str, List[Any]] = {}
        self._lock = threading.Lock()
        self._closed = False

    def _socket(self, addr: str):
        with self._lock:
            idle = self._idle.get(addr)
            if idle:
                return idle.pop()
        s = self._ctx.socket(zmq.REQ)
        for opt in (zmq.RCVTIMEO, zmq.SNDTIMEO):
            s.setsockopt(opt, self.timeout_ms)
        s.setsockopt(zmq.LINGER, 0)
        s.connect(f"tcp://{addr}")
        return s

    def call(self, addr: str, msg: dict) -> Optional[dict]:
        s = self._socket(addr)
        try:
            s.send(_pack(msg))
            reply = _unpack(s.recv())
        except zmq.ZMQError:
            s.close(0)
            return None
        except Exception as e:  # noqa: BLE001 - undecodable reply
            log.warning("PD: bad control reply from %s: %s", addr, e)
            s.close(0)
            return None
        with self._lock:
            if not self._closed:
                self._idle.setdefault(addr, []).append(s)
                return reply
        s.close(0)
        return reply

    def forget(self, addr: str) -> None:
        with self._lock:
            socks = self._idle.pop(addr, [])
        for s in socks:
            s.close(0)

    def close(self) -> None:
        with self._lock:
            self._closed = True
            idle, self._idle = self._idle, {}
        for socks in idle.values():
            for s in socks:
                s.close(0)


class _PullFailed(Exception):
    pass


class _PullJob:
    """One pull from one producer (one TP source when ``src`` is given)."""

    def __init__(self, consumer: "KVConsumer", req_id: str, addr: str, tid: str, local: List[int], first: int,
                 t0: float, src: Optional[TPSource]):
        self.c, self.req_id, self.addr, self.tid = consumer, req_id, addr, tid
        self.local, self.first, self.t0, self.src = local, first, t0, src

    def _acquire(self) -> dict:
        pause = 0.002
        while True:
            r = self.c.control(self.addr, {"op": "acquire", "tid": self.tid, "who": self.c.who})
            unknown = r is not None and not r.get("ok") and r.get("why") == "unknown"
            if not unknown or time.monotonic() - self.t0 > self.c.acquire_wait_s:
                break
            time.sleep(pause)                 # the hold may not have reached the producer yet
            pause = min(2 * pause, 0.05)
        if r is None:
            self.c.forget_peer(self.addr)
            raise _PullFailed("producer unreachable")
        if not r.get("ok"):
            raise _PullFailed(f"producer: {r.get('why')}")
        return r

    def _meta(self, inc: Optional[str]) -> _PeerMeta:
        meta = self.c.peer_meta(self.addr)
        if meta is not None and inc and meta.inc != inc:
            meta = self.c.peer_meta(self.addr, refresh=True)     # restarted at the same address
        if meta is None:
            raise _PullFailed("producer meta unavailable")
        if self.c.block_size and meta.block_size and meta.block_size != self.c.block_size:
            raise _PullFailed(f"block size {meta.block_size} != {self.c.block_size}")
        return meta

    def _plan(self, meta: _PeerMeta, remote: List[int]) -> list:
        s = self.src
        mine, theirs = self.c.layouts[0], meta.layouts[0]
        partial = s is not None and not (s.nheads == mine.heads == theirs.heads and mine.seg_bytes == theirs.seg_bytes
                                         and mine.head_stride == theirs.head_stride
                                         and mine.token_stride == theirs.token_stride)
        if partial:
            return head_read_ops(self.c.layouts, meta.layouts, self.local, remote, s.local_head0, s.remote_head0,
                                 s.nheads)
        return read_ops(self.c.layouts, meta.layouts, self.local, remote)

    def _read(self, meta: _PeerMeta, ops: list) -> None:
        st = self.c.staging
        rc = self.c.plane.read(meta.url, st.mirror_ops(ops) if st is not None else ops)
        if rc != 0:
            self.c.forget_peer(self.addr)
            raise _PullFailed(f"{self.c.plane.name} read returned {rc}")
        if st is not None:
            st.stage_in([(d, n) for d, _, n in ops])

    def run(self) -> PullResult:
        try:
            r = self._acquire()
            if not self.local:
                return PullResult(self.req_id, True)
            held = r["blocks"]
            remote = held[self.first:self.first + len(self.local)]
            if len(remote) < len(self.local):
                raise _PullFailed(f"producer holds {len(held)} blocks, need {self.first + len(self.local)}")
            meta = self._meta(r.get("inc"))
            ops = self._plan(meta, remote)
            outside = self.c.outside(ops)
            if outside:
                raise _PullFailed(f"read outside registered KV memory: {outside}")
            self._read(meta, ops)
            if self.c.release_after_pull:
                self.c.control(self.addr, self.c.release_msg(self.tid, self.src))
            return PullResult(self.req_id, True, nbytes=sum(n for _, _, n in ops),
                              seconds=time.monotonic() - self.t0)
        except _PullFailed as e:
            return PullResult(self.req_id, False, str(e))


class KVConsumer:
    def __init__(self, plane, layouts: Sequence[TensorLayout], block_size: int = 0, workers: int = 4,
                 ctrl_timeout_ms: int = 1000, register: bool = True, release_after_pull: bool = False,
                 acquire_wait_s: float = 2.0, device: str = "", who: str = ""):
        self.plane = plane
        self.device = device
        self.who = who or f"{os.getpid()}@{id(self):x}"
        self.inject_delay_s = float(os.getenv("CONNEX_PD_INJECT_PULL_DELAY_S", "0") or 0)
        self.acquire_wait_s = acquire_wait_s
        self.layouts = list(layouts)
        self.block_size = block_size
        self.release_after_pull = release_after_pull
        self.spans = register_spans(self.layouts)
        self.staging = register_with_staging(plane, self.spans, "KV consumer") if register \
            else getattr(plane, "_connex_staging", None)
        self._ctrl = _ControlPool(ctrl_timeout_ms)
        self._jobs = ThreadPoolExecutor(max_workers=workers, thread_name_prefix="connex-pd-pull")
        self._sources = ThreadPoolExecutor(max_workers=max(8, 2 * workers), thread_name_prefix="connex-pd-src")
        self._metas: Dict[str, _PeerMeta] = {}
        self._lock = threading.Lock()
        self._results: List[PullResult] = []
        self.stats = {"pulls": 0, "failed": 0, "bytes": 0, "seconds": 0.0}

    # ------------------------------------------------------------- control
    def control(self, addr: str, msg: dict) -> Optional[dict]:
        """One control request to the producer at ``addr`` (None on failure)."""
        return self._ctrl.call(addr, msg)

    def peer_meta(self, addr: str, refresh: bool = False) -> Optional[_PeerMeta]:
        with self._lock:
            cached = self._metas.get(addr)
        if cached is not None and not refresh:
            return cached
        r = self.control(addr, {"op": "meta"})
        if not r or not r.get("ok"):
            return None
        meta = _PeerMeta(r)
        if meta.spans is not None and hasattr(self.plane, "add_peer"):
            self.plane.add_peer(meta.url, meta.spans)
        with self._lock:
            self._metas[addr] = meta
        return meta

    def forget_peer(self, addr: str) -> None:
        with self._lock:
            self._metas.pop(addr, None)
        self._ctrl.forget(addr)

    def release_msg(self, tid: str, src: Optional[TPSource] = None) -> dict:
        m = {"op": "release", "tid": tid, "who": self.who}
        if src is not None and src.readers > 1:
            m["of"] = src.readers
        return m

    def outside(self, ops) -> Optional[tuple]:
        """The first destination not inside the registered KV memory, if any."""
        for dst, _, n in ops:
            if not any(s <= dst and dst + n <= s + ln for s, ln in self.spans):
                return hex(dst), n
        return None

    # ---------------------------------------------------------------- pulls
    def pull(self, req_id: str, addr: str, transfer_id: str, local_blocks: Sequence[int], first_block: int = 0,
             sources: Optional[Sequence[Tuple[str, TPSource]]] = None) -> None:
        """Start pulling remote blocks ``[first_block, +len(local_blocks))`` of
        ``transfer_id`` into ``local_blocks``; the outcome appears in
        :meth:`take_done`.  ``sources``: (address, TPSource) per remote TP rank."""
        self._jobs.submit(self._run, req_id, addr, transfer_id, list(local_blocks), first_block,
                          list(sources) if sources else None)

    def _run(self, req_id, addr, tid, local, first, sources) -> None:
        t0 = time.monotonic()
        try:
            if self.inject_delay_s:
                time.sleep(self.inject_delay_s)
            if sources:
                res = self._run_sources(req_id, sources, tid, local, first, t0)
            else:
                res = _PullJob(self, req_id, addr, tid, local, first, t0, None).run()
        except Exception as e:  # noqa: BLE001 - reported, never raised
            log.exception("KV pull of %s failed", req_id)
            res = PullResult(req_id, False, f"error: {e}")
        if not res.ok:
            res.failed_blocks = list(local)
        with self._lock:
            self.stats["pulls"] += 1
            self.stats["failed"] += not res.ok
            self.stats["bytes"] += res.nbytes
            self.stats["seconds"] += res.seconds
            self._results.append(res)

    def _run_sources(self, req_id, sources, tid, local, first, t0) -> PullResult:
        futs = [(a, s, self._sources.submit(_PullJob(self, req_id, a, tid, local, first, t0, s).run))
                for a, s in sources]
        total = 0
        for a, s, f in futs:
            r = f.result()
            if not r.ok:
                r.why = f"TP rank {s.remote_rank} ({a}): {r.why}"
                return r
            total += r.nbytes
        return PullResult(req_id, True, nbytes=total, seconds=time.monotonic() - t0)

    def release(self, addr: str, transfer_id: str, src: Optional[TPSource] = None) -> None:
        self._jobs.submit(self.control, addr, self.release_msg(transfer_id, src))

    def take_done(self) -> List[PullResult]:
        with self._lock:
            out, self._results = self._results, []
        return out

    def close(self) -> None:
        self._jobs.shutdown(wait=True)
        self._sources.shutdown(wait=True)
        self._ctrl.close()
