"""One-sided read transports for weight arenas (reference
``connex/rl/transport.py:44-251``).

Every transport has the same surface: ``url``, ``register(tensor) -> addr``,
``unregister``, ``read(url, addr, dst, dst_off, len)``, ``read_batch``,
``read_window`` (on failure the raised :class:`TransferError` carries
``done`` = leading ops that completed; reads are idempotent, so a caller
continues from there at another source), ``read_many`` and ``close``.

* :class:`LocalTransport` -- in-process owners, with ``kill()`` to simulate
  an owner's death (CPU tests, single-process benchmarks).
* :class:`NvlinkTransport` -- GPU arenas inside one NVLink/NVSwitch box:
  ``register`` exports the arena as a CUDA IPC handle into a per-owner record
  under ``/dev/shm``; a reader maps it once and pulls byte ranges with this
  package's SM copy kernel (one launch per batch, plain peer loads, no
  library kernel touches the peer's memory).  An owner whose process is gone
  or that called ``kill()`` is unreachable.
* :class:`EngineTransport` -- host (pinned) arenas across hosts through the
  native transfer engine (``connex_b200._cxengine``, TCP one-sided reads with
  heartbeats: a dead owner surfaces as an error within the per-op timeout).
"""
from __future__ import annotations

import json
import os
import socket
import threading
import uuid
from typing import Dict, List, Optional, Sequence, Tuple

import torch

Op = Tuple[int, int, int]   # (remote_addr, dst_off, length)


class TransferError(RuntimeError):
    done: int = 0


def advertise_ip() -> str:
    """``$CONNEX_ADVERTISE_IP``, else the address of this host's name, else loopback."""
    ip = os.environ.get("CONNEX_ADVERTISE_IP")
    if ip:
        return ip
    try:
        return socket.gethostbyname(socket.gethostname())
    except OSError:
        return "127.0.0.1"


def _nbytes(t: torch.Tensor) -> int:
    return t.numel() * t.element_size()


class _Counting:
    reads = 0
    bytes = 0

    def read(self, remote_url, remote_addr, dst, dst_off, length, timeout_ms=None):
        self.read_batch(remote_url, [(remote_addr, dst_off, length)], dst, timeout_ms)

    def read_many(self, remote_url, batches, timeout_ms=None):
        for dst, ops in batches:
            self.read_batch(remote_url, ops, dst, timeout_ms)

    def read_window(self, remote_url, ops, dst, window=16, timeout_ms=None):
        done = 0
        try:
            for i in range(0, len(ops), max(1, window)):
                part = ops[i:i + window]
                self.read_batch(remote_url, part, dst, timeout_ms)
                done += len(part)
        except TransferError as e:
            e.done = done
            raise


class LocalTransport(_Counting):
    """In-process owners: ``url -> {base_addr: uint8 tensor}``."""
    _owners: Dict[str, Dict[int, torch.Tensor]] = {}
    _dead: set = set()
    _lock = threading.Lock()

    def __init__(self, name: Optional[str] = None):
        self.url = f"local://{name or uuid.uuid4().hex[:8]}"
        with self._lock:
            self._owners[self.url] = {}
            self._dead.discard(self.url)
        self.reads = self.bytes = 0

    def register(self, tensor: torch.Tensor) -> int:
        with self._lock:
            self._owners[self.url][tensor.data_ptr()] = tensor.view(-1).view(torch.uint8)
        return tensor.data_ptr()

    def unregister(self, tensor: torch.Tensor) -> None:
        with self._lock:
            self._owners.get(self.url, {}).pop(tensor.data_ptr(), None)

    def _src(self, url: str, addr: int, n: int) -> torch.Tensor:
        with self._lock:
            if url in self._dead or url not in self._owners:
                raise TransferError(f"{url}: owner unreachable")
            for base, t in self._owners[url].items():
                if base <= addr and addr + n <= base + t.numel():
                    return t[addr - base:addr - base + n]
        raise TransferError(f"{url}: range [{addr:#x}, +{n}) not registered")

    def read_batch(self, remote_url, ops, dst, timeout_ms=None):
        flat = dst.view(-1).view(torch.uint8)
        for addr, off, n in ops:
            flat[off:off + n].copy_(self._src(remote_url, addr, n))
            self.reads += 1
            self.bytes += n

    def kill(self) -> None:
        with self._lock:
            self._dead.add(self.url)

    def close(self) -> None:
        with self._lock:
            self._owners.pop(self.url, None)


def _pid_alive(pid: int) -> bool:
    try:
        os.kill(pid, 0)
        return True
    except ProcessLookupError:
        return False
    except PermissionError:
        return True


class NvlinkTransport(_Counting):
    """GPU arenas over NVLink peer memory inside one box (CUDA IPC + copy kernel)."""

    def __init__(self, name: Optional[str] = None, device: Optional[int] = None, shm_dir: str = "/dev/shm"):
        self.device = torch.cuda.current_device() if device is None else device
        self.id = f"{os.getpid()}-{name or uuid.uuid4().hex[:8]}"
        self.url = f"nvlink://{socket.gethostname()}/{self.id}"
        self.dir = shm_dir
        self._regs: Dict[int, dict] = {}
        self._mappers: Dict[str, object] = {}
        self._lock = threading.Lock()
        self.reads = self.bytes = 0
        self._write_record()

    def _path(self, ident: str) -> str:
        return os.path.join(self.dir, f"connex-nvl-{ident}.json")

    def _write_record(self, dead: bool = False) -> None:
        rec = {"pid": os.getpid(), "dead": dead, "regions": list(self._regs.values())}
        tmp = self._path(self.id) + ".tmp"
        with open(tmp, "w") as f:
            json.dump(rec, f)
        os.replace(tmp, self._path(self.id))

    def register(self, tensor: torch.Tensor) -> int:
        from connex_b200.parallel.peer import export_tensor
        if not tensor.is_cuda:
            raise TransferError("NvlinkTransport registers GPU tensors only")
        h = export_tensor(tensor)
        with self._lock:
            self._regs[tensor.data_ptr()] = {"base": tensor.data_ptr(), "handle": h.handle.hex(),
                                             "offset": h.offset, "nbytes": h.nbytes, "device": h.owner_device}
            self._write_record()
        return tensor.data_ptr()

    def unregister(self, tensor: torch.Tensor) -> None:
        with self._lock:
            self._regs.pop(tensor.data_ptr(), None)
            self._write_record()

    def _resolve(self, url: str, addr: int, n: int) -> int:
        ident = url.rsplit("/", 1)[-1]
        try:
            with open(self._path(ident)) as f:
                rec = json.load(f)
        except (OSError, ValueError) as e:
            raise TransferError(f"{url}: no owner record ({e})") from None
        if rec["dead"] or not _pid_alive(rec["pid"]):
            raise TransferError(f"{url}: owner process gone")
        for r in rec["regions"]:
            if r["base"] <= addr and addr + n <= r["base"] + r["nbytes"]:
                if rec["pid"] == os.getpid():
                    return addr
                from connex_b200.parallel.peer import PeerHandle, PeerMapper
                with self._lock:
                    m = self._mappers.get(ident)
                    if m is None:
                        m = self._mappers[ident] = PeerMapper(self.device)
                local = m.open(PeerHandle(bytes.fromhex(r["handle"]), r["offset"], r["nbytes"], r["device"],
                                          rec["pid"]))
                return local + (addr - r["base"])
        raise TransferError(f"{url}: range [{addr:#x}, +{n}) not registered")

    def read_batch(self, remote_url, ops, dst, timeout_ms=None):
        from connex_b200 import ops as cx
        if not dst.is_cuda:
            raise TransferError("NvlinkTransport reads into GPU tensors only")
        base = dst.data_ptr()
        segs = [(self._resolve(remote_url, a, n), base + off, n) for a, off, n in ops]
        if not segs:
            return
        total = sum(s[2] for s in segs)
        with torch.cuda.device(dst.device):
            st = cx.new_status(dst.device)
            cx.copy_segments(torch.tensor(segs, dtype=torch.int64, device=dst.device), total, status=st)
            torch.cuda.current_stream(dst.device).synchronize()
            if int(st.item()) != 0:
                raise TransferError(f"{remote_url}: copy kernel status {int(st.item())}")
        self.reads += len(segs)
        self.bytes += total

    def read_many(self, remote_url, batches, timeout_ms=None):
        for dst, ops in batches:
            self.read_batch(remote_url, ops, dst, timeout_ms)

    def read_window(self, remote_url, ops, dst, window=16, timeout_ms=None):
        # one launch moves every chunk; a failure happens before any byte moved
        try:
            self.read_batch(remote_url, ops, dst, timeout_ms)
        except TransferError as e:
            e.done = 0
            raise

    def kill(self) -> None:
        with self._lock:
            self._write_record(dead=True)

    def close(self) -> None:
        for m in self._mappers.values():
            m.close()
        self._mappers.clear()
        try:
            os.unlink(self._path(self.id))
        except OSError:
            pass


class EngineTransport(_Counting):
    """Host arenas across hosts through the native transfer engine."""

    def __init__(self, lid=("connex-rl", 0, 0, 0), listen_ip: str = "0.0.0.0", port: int = 0,
                 advertise: Optional[str] = None, timeout_ms: int = 10000, engine=None):
        from connex_b200.engine import Engine
        model, stage, shard, replica = lid
        self.e = engine or Engine(model, stage, shard, replica, listen_ip=listen_ip, port=port,
                                  advertise_ip=advertise or advertise_ip())
        self.url = self.e.local_url
        self.timeout_ms = timeout_ms
        self.reads = self.bytes = 0

    def register(self, tensor: torch.Tensor) -> int:
        if tensor.is_cuda:
            raise TransferError("EngineTransport moves host memory; use a host arena")
        rc = self.e.register_memory(tensor.data_ptr(), _nbytes(tensor))
        if rc != 0:
            raise TransferError(f"register_memory failed: {rc}")
        return tensor.data_ptr()

    def unregister(self, tensor: torch.Tensor) -> None:
        self.e.unregister_memory(tensor.data_ptr())

    def read_batch(self, remote_url, ops, dst, timeout_ms=None):
        self.read_window(remote_url, ops, dst, window=len(ops) or 1, timeout_ms=timeout_ms)

    def read_window(self, remote_url, ops: Sequence[Op], dst, window=16, timeout_ms=None):
        """Up to ``window`` reads in flight; the next is posted as the oldest ends."""
        to = int(timeout_ms or self.timeout_ms)
        base = dst.data_ptr()
        inflight: List = []
        done = nxt = 0
        err: Optional[str] = None
        while (nxt < len(ops) or inflight) and err is None:
            while nxt < len(ops) and len(inflight) < window:
                a, off, n = ops[nxt]
                inflight.append(self.e.get_async(remote_url, base + off, a, n, to))
                nxt += 1
            rc = inflight.pop(0).wait(to + 1000)
            if rc != 0:
                err = f"read failed rc={rc} (-2 peer failed, -3 timeout, -4 invalid)"
            else:
                done += 1
        for h in inflight:      # posted reads must end before the caller reuses dst
            h.wait(to + 1000)
        self.reads += done
        self.bytes += sum(o[2] for o in ops[:done])
        if err is not None:
            e = TransferError(f"{remote_url}: {err}")
            e.done = done
            raise e

    def close(self) -> None:
        try:
            self.e.close()
        except Exception:  # noqa: BLE001
            pass


def make_transport(kind: Optional[str] = None, **kw):
    """``local`` | ``nvlink`` | ``engine`` (env ``CONNEX_RL_TRANSPORT``, default ``engine``)."""
    kind = kind or os.environ.get("CONNEX_RL_TRANSPORT", "engine")
    if kind == "local":
        return LocalTransport(kw.get("name"))
    if kind == "nvlink":
        return NvlinkTransport(kw.get("name"), kw.get("device"))
    return EngineTransport(**{k: v for k, v in kw.items() if k not in ("name", "device")})
