"""Elastic point-to-point activation links between pipeline stage processes.

Pipeline activations (``[batch, hidden]`` bf16 per hop) travel over NCCL
send/recv, but a fixed NCCL world cannot lose or gain a member.  Here every
direction between two stage endpoints that talk gets its own two-rank
process group, created on demand: both sides rendezvous through a shared
``TCPStore`` under the prefix ``cxpp/<sender>><receiver>/<generation>``
(rank 0 = sender).  One group per direction keeps a stage's forward sends
and its reply receives on different NCCL streams, so K steps in flight in
both directions cannot wait on each other.  When a peer dies only its
groups are aborted; a replacement opens fresh ones (a new generation when
it reuses the name).  The same code runs on ``gloo`` (CPU tests).

Sends and receives run on a dedicated CUDA stream per link so they overlap
the stage's compute; the caller orders them with events.  Which peer to talk
to, and when a peer is dead, is decided by the control plane (directory /
front-router routes and the step protocol), never by this module.
"""
from __future__ import annotations

import threading
from datetime import timedelta
from typing import Dict, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist


class LinkError(RuntimeError):
    pass


class PairLink:
    def __init__(self, me: str, peer: str, gen: int, pg, rank: int, device: torch.device):
        self.me, self.peer, self.gen = me, peer, gen
        self.pg = pg
        self.rank = rank
        self.peer_rank = 1 - rank
        self.device = device
        self.stream = torch.cuda.Stream(device) if device.type == "cuda" else None
        self.sent = self.received = 0
        self.dead = False

    def _run(self, fn, tensors: Sequence[torch.Tensor], after: Optional[torch.cuda.Event]):
        if self.dead:
            raise LinkError(f"link {self.me}->{self.peer} (gen {self.gen}) is closed")
        if self.stream is None:
            works = [fn(t) for t in tensors]
            for w in works:
                w.wait()
            return works
        cur = torch.cuda.current_stream(self.device)
        self.stream.wait_stream(cur) if after is None else self.stream.wait_event(after)
        with torch.cuda.device(self.device), torch.cuda.stream(self.stream):
            works = [fn(t) for t in tensors]
            for w in works:       # the link stream (not the host) waits for the NCCL stream
                w.wait()
        for t in tensors:
            t.record_stream(self.stream)
        return works

    def send(self, tensors: Sequence[torch.Tensor], after: Optional[torch.cuda.Event] = None):
        """Post sends of ``tensors`` (in order); returns the works."""
        works = self._run(lambda t: self.pg.send([t], self.peer_rank, 0), tensors, after)
        self.sent += len(tensors)
        return works

    def recv(self, tensors: Sequence[torch.Tensor]):
        """Post receives into ``tensors`` (same order as the peer's sends)."""
        works = self._run(lambda t: self.pg.recv([t], self.peer_rank, 0), tensors, None)
        self.received += len(tensors)
        return works

    def done_event(self) -> Optional[torch.cuda.Event]:
        """Event after everything posted so far on the link's stream."""
        if self.stream is None:
            return None
        ev = torch.cuda.Event()
        ev.record(self.stream)
        return ev

    def close(self, abort: bool = False) -> None:
        if self.dead:
            return
        self.dead = True
        try:
            if abort and hasattr(self.pg, "abort"):
                self.pg.abort()
            elif hasattr(self.pg, "shutdown"):
                self.pg.shutdown()
        except Exception:  # noqa: BLE001 - a dead peer's group may refuse a clean shutdown
            pass


class PairLinks:
    """All pair links of one stage endpoint (``me``)."""

    def __init__(self, store: dist.Store, me: str, device, backend: Optional[str] = None, timeout_s: float = 30.0):
        self.store = store
        self.me = me
        self.device = torch.device(device)
        self.backend = backend or ("nccl" if self.device.type == "cuda" else "gloo")
        self.timeout = timedelta(seconds=timeout_s)
        self.links: Dict[Tuple[str, int, bool], PairLink] = {}
        self._lock = threading.Lock()

    @staticmethod
    def prefix(sender: str, receiver: str, gen: int) -> str:
        return f"cxpp/{sender}>{receiver}/{gen}/"

    def open_tx(self, peer: str, gen: int = 0) -> PairLink:
        """Link for sending to ``peer`` (which opens it with ``open_rx(me, gen)``)."""
        return self._open(peer, gen, True)

    def open_rx(self, peer: str, gen: int = 0) -> PairLink:
        """Link for receiving from ``peer`` (which opens it with ``open_tx(me, gen)``)."""
        return self._open(peer, gen, False)

    def _open(self, peer: str, gen: int, tx: bool) -> PairLink:
        key = (peer, gen, tx)
        with self._lock:
            link = self.links.get(key)
            if link is not None and not link.dead:
                return link
        if peer == self.me:
            raise ValueError("a link needs two endpoints")
        rank = 0 if tx else 1
        pstore = dist.PrefixStore(self.prefix(self.me, peer, gen) if tx else self.prefix(peer, self.me, gen),
                                  self.store)
        if self.backend == "nccl":
            opts = dist.ProcessGroupNCCL.Options()
            opts._timeout = self.timeout
            pg = dist.ProcessGroupNCCL(pstore, rank, 2, opts)
        else:
            pg = dist.ProcessGroupGloo(pstore, rank, 2, self.timeout)
        link = PairLink(self.me, peer, gen, pg, rank, self.device)
        with self._lock:
            self.links[key] = link
        return link

    def get(self, peer: str, gen: int = 0, tx: bool = True) -> Optional[PairLink]:
        return self.links.get((peer, gen, tx))

    def drop_peer(self, peer: str, abort: bool = True) -> int:
        """Close every link to ``peer`` (it died or left); returns how many."""
        with self._lock:
            keys = [k for k in self.links if k[0] == peer]
            links = [self.links.pop(k) for k in keys]
        for l in links:
            l.close(abort=abort)
        return len(links)

    def close(self) -> None:
        with self._lock:
            links = list(self.links.values())
            self.links.clear()
        for l in links:
            l.close()


def tensor_specs(td: dict) -> List[Tuple[str, torch.dtype, tuple]]:
    """Ordered ``(key, dtype, shape)`` of the tensors of a tensor dict."""
    return [(k, v.dtype, tuple(v.shape)) for k, v in td.items() if isinstance(v, torch.Tensor)]


def alloc_like(specs, device) -> Dict[str, torch.Tensor]:
    return {k: torch.empty(s, dtype=d, device=device) for k, d, s in specs}
