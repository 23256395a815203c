"""Pull-based KV block transfer between a prefill and a decode instance.

Prefill side :class:`KVProducer`: after a request's prefill it *holds* the
KV blocks under a transfer id (a lease renewed by every acquire, freed after
``retain_s`` without one) and serves a ZeroMQ ROUTER control channel with
msgpack ops (the reference's ``connex/pd/transfer.py:148-195``):

* ``{"op": "meta"}``    -> incarnation, data-plane URL / backend, engine id,
  block size, device, KV layouts (and, for the NVLink plane, the IPC spans);
* ``{"op": "acquire", "tid", "who"}`` -> the held block ids (renews the lease);
* ``{"op": "release", "tid", "who", ["of"]}`` -> frees once all ``of`` readers
  released (stale-owner guard for single-reader releases);
* ``{"op": "ping"}``.

Decode side :class:`KVConsumer`: acquires (retrying while the hold is still
unknown), fetches / caches the producer's meta by incarnation, builds the
fewest one-sided reads (``read_ops`` / ``head_read_ops`` for heterogeneous
TP), checks that every destination lies in its registered KV memory, reads
through its data plane, and reports a per-request :class:`PullResult` --
failures are reported, never raised.  Holding until release (not freeing
after the first read) lets a replacement decode instance re-pull the prompt
KV after a decode death instead of re-running prefill.
"""
from __future__ import annotations

import logging
import os
import threading
import time
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, field
from typing import List, Optional, Sequence, Tuple

import msgpack
import zmq

from connex.pd.dataplane import ZCOPY_THRESH
from connex.pd.host_staging import block_ranges, register_with_staging
from connex.pd.kv_layout import TPSource, TensorLayout, head_read_ops, read_ops, register_spans

log = logging.getLogger("connex.pd")
PROTO_VERSION = 1


def _pack(o) -> bytes:
    return msgpack.packb(o, use_bin_type=True)


def _unpack(b: bytes):
    return msgpack.unpackb(b, raw=False)


@dataclass
class _Hold:
    req_id: str
    blocks: List[int]
    deadline: float
    acquired: int = 0
    released_by: set = field(default_factory=set)
    ready: object = None
    owner: object = None


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
        self._holds: dict = {}
        self._released: set = set()
        self._finished: set = set()
        self._lock = threading.Lock()
        self.stats = {"holds": 0, "acquires": 0, "releases": 0, "expired": 0, "unknown": 0}
        self._staging = register_with_staging(plane, register_spans(self.layouts), "KV producer") if register \
            else getattr(plane, "_connex_staging", None)
        self._sock = zmq.Context.instance().socket(zmq.ROUTER)
        self._sock.setsockopt(zmq.LINGER, 0)
        if port:
            self._sock.bind(f"tcp://{bind_ip}:{port}")
            self.port = port
        else:
            self.port = self._sock.bind_to_random_port(f"tcp://{bind_ip}")
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._serve, name="connex-pd-producer", daemon=True)
        self._thread.start()

    # ------------------------------------------------------------- engine
    def hold(self, req_id: str, transfer_id: str, blocks: Sequence[int]) -> None:
        with self._lock:
            if transfer_id in self._released:  # released before the hold arrived
                self._released.discard(transfer_id)
                self._finished.add(req_id)
                return
        ready = self._staging.stage_out(block_ranges(self.layouts, blocks)) if self._staging is not None else None
        with self._lock:
            self._holds[transfer_id] = _Hold(req_id, list(blocks), time.monotonic() + self.retain_s, ready=ready)
            self.stats["holds"] += 1

    def drop(self, transfer_id: str) -> None:
        with self._lock:
            self._holds.pop(transfer_id, None)

    def take_finished(self) -> set:
        """Request ids whose blocks may be freed now (released or lease expired)."""
        now = time.monotonic()
        with self._lock:
            for tid, h in list(self._holds.items()):
                if h.deadline < now:
                    del self._holds[tid]
                    self._finished.add(h.req_id)
                    self.stats["expired"] += 1
            out, self._finished = self._finished, set()
        return out

    def held(self) -> int:
        with self._lock:
            return len(self._holds)

    # ----------------------------------------------------------- control
    def _meta(self) -> dict:
        d = {"ok": True, "v": PROTO_VERSION, "inc": self.inc, "url": self.plane.local_url,
             "backend": self.plane.name, "engine_id": self.engine_id, "block_size": self.block_size,
             "device": self.device,
             "layouts": [(self._staging.translate(lo) if self._staging else lo).to_dict() for lo in self.layouts]}
        describe = getattr(self.plane, "describe", None)
        if describe is not None and self._staging is None:
            d["spans"] = describe()
        return d

    def _handle(self, m: dict) -> dict:
        op = m.get("op")
        if op == "meta":
            return self._meta()
        tid = m.get("tid")
        with self._lock:
            h = self._holds.get(tid)
            if op == "acquire":
                if h is None:
                    self.stats["unknown"] += 1
                    return {"ok": False, "why": "unknown"}
                h.acquired += 1
                if m.get("who"):
                    h.owner = m.get("who")
                h.deadline = time.monotonic() + self.retain_s
                self.stats["acquires"] += 1
                return {"ok": True, "blocks": h.blocks, "inc": self.inc, "_wait": h.ready}
            if op == "release":
                self.stats["releases"] += 1
                of, who = int(m.get("of") or 1), m.get("who")
                if h is not None and of <= 1 and who and h.owner and who != h.owner:
                    self.stats["stale_releases"] = self.stats.get("stale_releases", 0) + 1
                    return {"ok": True, "stale": True}
                if h is not None and of > 1:
                    h.released_by.add(who)
                    if len(h.released_by) < of:
                        return {"ok": True, "pending": of - len(h.released_by)}
                if h is None:
                    self._released.add(tid)
                    if len(self._released) > 100000:
                        self._released.clear()
                else:
                    del self._holds[tid]
                    self._finished.add(h.req_id)
                return {"ok": True}
            if op == "ping":
                return {"ok": True, "held": len(self._holds)}
        return {"ok": False, "why": f"bad op {op!r}"}

    @staticmethod
    def _ready(ev) -> bool:
        try:
            return bool(ev.query())
        except Exception:
            ev.synchronize()
            return True

    def _serve(self) -> None:
        poller = zmq.Poller()
        poller.register(self._sock, zmq.POLLIN)
        waiting: list = []  # replies whose staged copy has not finished
        while not self._stop.is_set():
            if poller.poll(1 if waiting else 100):
                frames = self._sock.recv_multipart()
                env, body = frames[:-1], frames[-1]
                try:
                    rep = self._handle(_unpack(body))
                    ev = rep.pop("_wait", None)
                except Exception as e:
                    rep, ev = {"ok": False, "why": f"error: {e}"}, None
                if ev is not None and not self._ready(ev):
                    waiting.append((ev, env, rep))
                else:
                    self._sock.send_multipart(env + [_pack(rep)])
            if waiting:
                still = []
                for ev, env, rep in waiting:
                    if self._ready(ev):
                        self._sock.send_multipart(env + [_pack(rep)])
                    else:
                        still.append((ev, env, rep))
                waiting = still

    def close(self) -> None:
        self._stop.set()
        self._thread.join(timeout=2)
        self._sock.close(0)


@dataclass
class PullResult:
    req_id: str
    ok: bool
    why: str = ""
    nbytes: int = 0
    seconds: float = 0.0
    failed_blocks: List[int] = field(default_factory=list)


class _PeerMeta:
    def __init__(self, d: dict):
        self.url = d["url"]
        self.backend = d.get("backend")
        self.engine_id = d.get("engine_id")
        self.inc = d.get("inc")
        self.block_size = d.get("block_size", 0)
        self.device = d.get("device", "")
        self.layouts = [TensorLayout.from_dict(x) for x in d["layouts"]]
        self.spans = d.get("spans")


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
        self.ctrl_timeout_ms = ctrl_timeout_ms
        self.release_after_pull = release_after_pull
        self._spans = register_spans(self.layouts)
        self._staging = register_with_staging(plane, self._spans, "KV consumer") if register \
            else getattr(plane, "_connex_staging", None)
        self._pool = ThreadPoolExecutor(max_workers=workers, thread_name_prefix="connex-pd-pull")
        self._src_pool = ThreadPoolExecutor(max_workers=max(8, 2 * workers), thread_name_prefix="connex-pd-src")
        self._meta: dict = {}
        self._lock = threading.Lock()
        self._done: List[PullResult] = []
        self._ctx = zmq.Context.instance()
        self._socks: dict = {}
        self._closed = False
        self.stats = {"pulls": 0, "failed": 0, "bytes": 0, "seconds": 0.0}

    # ------------------------------------------------------------ control
    def _call(self, addr: str, msg: dict) -> Optional[dict]:
        with self._lock:
            idle = self._socks.get(addr)
            s = idle.pop() if idle else None
        if s is None:
            s = self._ctx.socket(zmq.REQ)
            s.setsockopt(zmq.LINGER, 0)
            s.setsockopt(zmq.RCVTIMEO, self.ctrl_timeout_ms)
            s.setsockopt(zmq.SNDTIMEO, self.ctrl_timeout_ms)
            s.connect(f"tcp://{addr}")
        try:
            s.send(_pack(msg))
            rep = _unpack(s.recv())
        except Exception as e:
            s.close(0)
            if not isinstance(e, zmq.ZMQError):
                log.warning("PD: bad control reply from %s: %s", addr, e)
            return None
        with self._lock:
            if not self._closed:
                self._socks.setdefault(addr, []).append(s)
                s = None
        if s is not None:
            s.close(0)
        return rep

    def peer_meta(self, addr: str, refresh: bool = False) -> Optional[_PeerMeta]:
        with self._lock:
            m = self._meta.get(addr)
        if m is not None and not refresh:
            return m
        r = self._call(addr, {"op": "meta"})
        if not r or not r.get("ok"):
            return None
        m = _PeerMeta(r)
        if m.spans is not None and hasattr(self.plane, "add_peer"):
            self.plane.add_peer(m.url, m.spans)
        with self._lock:
            self._meta[addr] = m
        return m

    def forget_peer(self, addr: str) -> None:
        with self._lock:
            self._meta.pop(addr, None)
            socks = self._socks.pop(addr, [])
        for s in socks:
            s.close(0)

    # --------------------------------------------------------------- pull
    def pull(self, req_id: str, addr: str, transfer_id: str, local_blocks: Sequence[int], first_block: int = 0,
             sources: Optional[Sequence[Tuple[str, TPSource]]] = None) -> None:
        """Start pulling remote blocks [first_block, +len(local)) of
        ``transfer_id`` into ``local_blocks``; the result shows up in ``take_done``."""
        self._pool.submit(self._pull, req_id, addr, transfer_id, list(local_blocks), first_block,
                          list(sources) if sources else None)

    def _pull(self, req_id, addr, tid, local, first, sources=None) -> None:
        t0 = time.monotonic()
        res = PullResult(req_id, False, failed_blocks=local)
        try:
            res = self._pull_sources(req_id, sources, tid, local, first, t0) if sources else \
                self._pull_inner(req_id, addr, tid, local, first, t0)
        except Exception as e:
            res.why = f"error: {e}"
            log.exception("KV pull of %s failed", req_id)
        if not res.ok:
            res.failed_blocks = list(local)
        with self._lock:
            self.stats["pulls"] += 1
            self.stats["failed"] += 0 if res.ok else 1
            self.stats["bytes"] += res.nbytes
            self.stats["seconds"] += res.seconds
            self._done.append(res)

    def _pull_sources(self, req_id, sources, tid, local, first, t0) -> PullResult:
        if self.inject_delay_s:
            time.sleep(self.inject_delay_s)
        futs = [self._src_pool.submit(self._pull_inner, req_id, a, tid, local, first, t0, src=s, delay=False)
                for a, s in sources]
        nbytes = 0
        for (a, s), f in zip(sources, futs):
            r = f.result()
            if not r.ok:
                r.why = f"TP rank {s.remote_rank} ({a}): {r.why}"
                return r
            nbytes += r.nbytes
        return PullResult(req_id, True, nbytes=nbytes, seconds=time.monotonic() - t0)

    def _pull_inner(self, req_id, addr, tid, local, first, t0, src: Optional[TPSource] = None,
                    delay: bool = True) -> PullResult:
        if self.inject_delay_s and delay:
            time.sleep(self.inject_delay_s)
        backoff = 0.002
        while True:
            r = self._call(addr, {"op": "acquire", "tid": tid, "who": self.who})
            if r is None or r.get("ok") or r.get("why") != "unknown" or time.monotonic() - t0 > self.acquire_wait_s:
                break
            time.sleep(backoff)
            backoff = min(backoff * 2, 0.05)
        if r is None:
            self.forget_peer(addr)
            return PullResult(req_id, False, "producer unreachable")
        if not r.get("ok"):
            return PullResult(req_id, False, f"producer: {r.get('why')}")
        if not local:
            return PullResult(req_id, True)
        remote = r["blocks"][first:first + len(local)]
        if len(remote) < len(local):
            return PullResult(req_id, False, f"producer holds {len(r['blocks'])} blocks, need {first + len(local)}")
        meta = self.peer_meta(addr)
        if meta is not None and r.get("inc") and meta.inc != r["inc"]:
            meta = self.peer_meta(addr, refresh=True)  # restarted at the same address
        if meta is None:
            return PullResult(req_id, False, "producer meta unavailable")
        if self.block_size and meta.block_size and meta.block_size != self.block_size:
            return PullResult(req_id, False, f"block size {meta.block_size} != {self.block_size}")
        ops = self._ops(meta, local, remote, src)
        if self.plane.name == "cxengine" and self._staging is None and ops and \
                min(n for _, _, n in ops) < ZCOPY_THRESH:
            log.debug("KV segment below %d B: small reads", ZCOPY_THRESH)
        bad = self._outside(ops)
        if bad:
            return PullResult(req_id, False, f"read outside registered KV memory: {bad}")
        if self._staging is not None:
            rc = self.plane.read(meta.url, self._staging.mirror_ops(ops))
            if rc == 0:
                self._staging.stage_in([(d, n) for d, _, n in ops])
        else:
            rc = self.plane.read(meta.url, ops)
        if rc != 0:
            self.forget_peer(addr)
            return PullResult(req_id, False, f"{self.plane.name} read returned {rc}")
        if self.release_after_pull:
            self._call(addr, self._release_msg(tid, src))
        return PullResult(req_id, True, nbytes=sum(n for _, _, n in ops), seconds=time.monotonic() - t0)

    def _ops(self, meta: _PeerMeta, local, remote, src: Optional[TPSource]):
        if src is not None:
            lo, ro = self.layouts[0], meta.layouts[0]
            whole = (src.nheads == lo.heads == ro.heads and lo.seg_bytes == ro.seg_bytes
                     and lo.head_stride == ro.head_stride and lo.token_stride == ro.token_stride)
            if not whole:
                return head_read_ops(self.layouts, meta.layouts, local, remote, src.local_head0, src.remote_head0,
                                     src.nheads)
        return read_ops(self.layouts, meta.layouts, local, remote)

    def _release_msg(self, tid: str, src: Optional[TPSource] = None) -> dict:
        m = {"op": "release", "tid": tid, "who": self.who}
        if src is not None and src.readers > 1:
            m["of"] = src.readers
        return m

    def _outside(self, ops) -> Optional[tuple]:
        for dst, _, n in ops:
            if not any(s <= dst and dst + n <= s + ln for s, ln in self._spans):
                return (hex(dst), n)
        return None

    def release(self, addr: str, transfer_id: str, src: Optional[TPSource] = None) -> None:
        self._pool.submit(self._call, addr, self._release_msg(transfer_id, src))

    def take_done(self) -> List[PullResult]:
        with self._lock:
            out, self._done = self._done, []
        return out

    def close(self) -> None:
        self._pool.shutdown(wait=True)
        self._src_pool.shutdown(wait=True)
        with self._lock:
            self._closed = True
            socks, self._socks = self._socks, {}
        for lst in socks.values():
            for s in lst:
                s.close(0)
