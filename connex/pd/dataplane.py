"""Data planes for PD KV transfer: register memory, batched one-sided reads.

A plane registers the KV cache, tells peers how to reach it (``local_url``)
and reads a batch of ``(dst, src, length)`` ranges from a peer, returning 0
or a negative code (``PEER_FAILED`` -2, ``TIMEOUT`` -3, ``INVALID`` -4; the
codes of ``connex/pd/dataplane.py:29-32`` in the reference).

* :class:`NVLinkPlane` -- GPU memory inside one NVLink/NVSwitch box: spans
  are exported as CUDA IPC handles (``describe()``, sent in the producer's
  ``meta`` reply), the reader maps them once and moves every batch with one
  launch of this package's ``copy_segments`` kernel (SM loads over NVLink).
* :class:`CxEnginePlane` -- the native transfer engine (TCP, host memory):
  every read of a batch is posted (``get_async``) and then waited for.
* :class:`LoopbackPlane` -- same-process ``memmove`` of host memory (tests).

``make_plane`` picks one from ``CONNEX_PD_BACKEND`` (``auto`` | ``nvlink`` |
``cxengine`` | ``loopback``; ``connex-rs`` / ``mooncake`` are accepted as
aliases of ``cxengine``, whose surface they share).
"""
from __future__ import annotations

import ctypes
import logging
import os
import threading
from typing import List, Optional, Protocol, Sequence, Tuple

log = logging.getLogger("connex.pd")

ZCOPY_THRESH = 4096
PEER_FAILED = -2
TIMEOUT = -3
INVALID = -4

Op = Tuple[int, int, int]


def setup_ucx_env(ip: str) -> None:
    """Environment defaults kept for parity with UCX-based deployments:
    zero-copy threshold pinned below a KV block and CUDA-IPC through UCX off
    (explicit settings win).  Inside one box the NVLink plane is used."""
    os.environ.setdefault("UCX_TCP_CM_REUSEADDR", "y")
    os.environ.setdefault("UCX_ZCOPY_THRESH", str(ZCOPY_THRESH))
    if os.getenv("CONNEX_RS_CUDA_IPC", "0") != "1" and not os.getenv("UCX_TLS"):
        os.environ["UCX_TLS"] = "^cuda_ipc"


class KVDataPlane(Protocol):
    name: str
    local_url: str

    def register(self, ptr: int, length: int) -> int: ...

    def unregister(self, ptr: int) -> int: ...

    def read(self, peer_url: str, ops: Sequence[Op]) -> int: ...

    def close(self) -> None: ...


def is_device_ptr(ptr: int) -> bool:
    """True if ``ptr`` is CUDA device memory (False without a CUDA runtime)."""
    try:
        import torch
        if not torch.cuda.is_available():
            return False
        from connex_b200 import _C  # noqa: F401  (CUDA runtime is loaded with it)
        lib = ctypes.CDLL("libcudart.so.12") if os.path.exists("/usr/local/cuda/lib64/libcudart.so.12") else None
        if lib is None:
            return False

        class Attr(ctypes.Structure):
            _fields_ = [("type", ctypes.c_int), ("device", ctypes.c_int), ("devicePointer", ctypes.c_void_p),
                        ("hostPointer", ctypes.c_void_p)]
        a = Attr()
        if lib.cudaPointerGetAttributes(ctypes.byref(a), ctypes.c_void_p(ptr)) != 0:
            lib.cudaGetLastError()
            return False
        return a.type in (2, 3)  # device, managed
    except Exception:
        return False


class LoopbackPlane:
    """Same-process memmove of host memory (tests only)."""

    name = "loopback"

    def __init__(self, *_, **__):
        self.local_url = f"loopback://{os.getpid()}"
        self.spans: List[Tuple[int, int]] = []
        self.reads = 0
        self._lock = threading.Lock()

    def register(self, ptr: int, length: int) -> int:
        self.spans.append((ptr, length))
        return 0

    def unregister(self, ptr: int) -> int:
        self.spans = [s for s in self.spans if s[0] != ptr]
        return 0

    def read(self, peer_url: str, ops: Sequence[Op]) -> int:
        with self._lock:
            for dst, src, n in ops:
                ctypes.memmove(dst, src, n)
            self.reads += 1
        return 0

    def close(self) -> None:
        pass


class CxEnginePlane:
    """The native transfer engine: batched ``get_async`` then wait all."""

    name = "cxengine"

    def __init__(self, model: str, role_idx: int, replica: int, rank: int, ip: str = "127.0.0.1", port: int = 0,
                 timeout_ms: int = 10000):
        from connex_b200.engine import Engine
        self.engine = Engine(model, role_idx, rank, replica, listen_ip=ip, port=port)
        self.local_url = self.engine.local_url
        self.timeout_ms = timeout_ms

    def register(self, ptr: int, length: int) -> int:
        return self.engine.register_memory(ptr, length)

    def unregister(self, ptr: int) -> int:
        return self.engine.unregister_memory(ptr)

    def read(self, peer_url: str, ops: Sequence[Op]) -> int:
        hs = [self.engine.get_async(peer_url, d, s, n, self.timeout_ms) for d, s, n in ops]
        rc = 0
        for h in hs:
            r = h.wait(self.timeout_ms)
            if r != 0 and rc == 0:
                rc = r
        return rc

    def close(self) -> None:
        self.engine.close()


class NVLinkPlane:
    """GPU KV inside one NVLink box, read with SM copy kernels over peer mappings."""

    name = "nvlink"

    def __init__(self, device: Optional[int] = None, **_):
        import torch
        self.torch = torch
        self.device = torch.cuda.current_device() if device is None else device
        self.local_url = f"nvlink://{os.uname().nodename}/{os.getpid()}/{self.device}"
        self._spans: List[Tuple[int, int]] = []
        self._peers: dict = {}      # url -> [(remote base, length, local mapped base)]
        self._lock = threading.Lock()
        from connex_b200.parallel.peer import PeerMapper
        self._mapper = PeerMapper(self.device)
        self._stream = torch.cuda.Stream(device=self.device)
        self.reads = 0

    def register(self, ptr: int, length: int) -> int:
        self._spans.append((ptr, length))
        return 0

    def unregister(self, ptr: int) -> int:
        n = len(self._spans)
        self._spans = [s for s in self._spans if s[0] != ptr]
        return 0 if len(self._spans) < n else INVALID

    def describe(self) -> List[dict]:
        """IPC handles of the registered spans (sent to readers)."""
        from connex_b200 import ops
        out = []
        for ptr, n in self._spans:
            h, off = ops.ipc_export(ptr, self.device)
            out.append({"base": ptr, "len": n, "handle": h, "offset": off, "pid": os.getpid()})
        return out

    def add_peer(self, peer_url: str, spans: List[dict]) -> None:
        from connex_b200.parallel.peer import PeerHandle
        mapped = []
        for s in spans:
            if int(s.get("pid", -1)) == os.getpid():
                mapped.append((s["base"], s["len"], s["base"]))
            else:
                addr = self._mapper.open(PeerHandle(bytes(s["handle"]), int(s["offset"]), int(s["len"]),
                                                    -1, int(s["pid"])))
                mapped.append((s["base"], s["len"], addr))
        with self._lock:
            self._peers[peer_url] = mapped

    def _translate(self, peer_url: str, src: int, n: int) -> Optional[int]:
        for base, ln, local in self._peers.get(peer_url, ()):
            if base <= src and src + n <= base + ln:
                return local + (src - base)
        return None

    def read(self, peer_url: str, ops: Sequence[Op]) -> int:
        from connex_b200 import ops as cxops
        torch = self.torch
        segs = []
        total = 0
        for d, s, n in ops:
            m = self._translate(peer_url, s, n)
            if m is None:
                return INVALID
            segs.append((m, d, n))
            total += n
        if not segs:
            return 0
        with torch.cuda.device(self.device), torch.cuda.stream(self._stream):
            st = cxops.new_status(self.device)
            t = torch.tensor(segs, dtype=torch.int64).to(f"cuda:{self.device}", non_blocking=True)
            cxops.copy_segments(t, total, status=st)
            self._stream.synchronize()
            code = int(st.item())
        self.reads += 1
        return 0 if code == 0 else INVALID

    def close(self) -> None:
        self._mapper.close()


def backend_from_env() -> str:
    return resolve_backend(os.getenv("CONNEX_PD_BACKEND"))


def resolve_backend(name: Optional[str]) -> str:
    n = (name or "auto").strip().lower().replace("_", "-")
    if n in ("connex-rs", "connexrs", "mooncake", "cx", "cxengine", "tcp"):
        return "cxengine"
    if n in ("nvlink", "ipc", "p2p"):
        return "nvlink"
    if n == "loopback":
        return "loopback"
    if n == "auto":
        try:
            import torch
            return "nvlink" if torch.cuda.is_available() else "cxengine"
        except Exception:
            return "cxengine"
    raise ValueError(f"unknown PD data plane {name!r} (auto | nvlink | cxengine | loopback)")


def make_plane(model: str, role_idx: int, replica: int, rank: int, ip: str = "127.0.0.1",
               backend: Optional[str] = None, device: Optional[int] = None):
    b = resolve_backend(backend or os.getenv("CONNEX_PD_BACKEND"))
    if b == "nvlink":
        return NVLinkPlane(device=device)
    if b == "loopback":
        return LoopbackPlane()
    setup_ucx_env(ip)
    return CxEnginePlane(model, role_idx, replica, rank, ip=ip)
