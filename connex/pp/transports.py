"""Data-plane selection for pipeline endpoints (reference ``connex/pp/transports.py:52-315``).

A message moves as: the sender stages the tensors, sends a small ZeroMQ
signal (:mod:`connex.pp.wire`), the receiver fetches the bytes.  Backends:

* ``nccl`` -- device activations over elastic two-rank NCCL groups
  (:mod:`connex_b200.parallel.pplink`), the path inside one NVLink box;
* ``cxengine`` -- the native transfer engine (``connex_b200._cxengine``):
  one-sided reads of a registered host send ring, peer-failure events,
  same-identity rejoin; ``connex-rs`` / ``rs`` are aliases (same surface);
* ``zmq`` -- bytes inline in the ZeroMQ message.

``mooncake`` is accepted as a name but is not part of this build: it raises
with a pointer to ``cxengine``.
"""
from __future__ import annotations

import logging
import os
from typing import Optional, Protocol

BACKENDS = ("nccl", "cxengine", "zmq")
ALIASES = {"connex-rs": "cxengine", "connexrs": "cxengine", "connex_rs": "cxengine", "rs": "cxengine",
           "none": "zmq", "zeromq": "zmq", "gloo": "nccl"}
DEFAULT_BACKEND = "auto"


def native_engine_available() -> bool:
    try:
        import connex_b200._cxengine  # noqa: F401
        return True
    except ImportError:
        return False


def backend_from_env(has_cuda: Optional[bool] = None) -> str:
    """``CONNEX_PP_BACKEND``: nccl | cxengine | zmq | auto (default: nccl with
    CUDA, else cxengine when the native module is built, else zmq)."""
    b = (os.getenv("CONNEX_PP_BACKEND") or DEFAULT_BACKEND).strip().lower()
    b = ALIASES.get(b, b)
    if b == "mooncake":
        raise ValueError("the Mooncake transfer engine is not part of this build; use CONNEX_PP_BACKEND=cxengine "
                         "(same one-sided read surface) or nccl")
    if b == "auto":
        if has_cuda is None:
            try:
                import torch
                has_cuda = torch.cuda.is_available()
            except ImportError:
                has_cuda = False
        if has_cuda:
            return "nccl"
        return "cxengine" if native_engine_available() else "zmq"
    if b not in BACKENDS:
        raise ValueError(f"CONNEX_PP_BACKEND must be one of {BACKENDS} or auto, got {b!r}")
    return b


class TransferEngine(Protocol):
    """The one-sided transfer surface the endpoint uses."""

    def allocate_managed_buffer(self, size: int) -> int: ...
    def free_managed_buffer(self, ptr: int, size: int) -> None: ...
    def write_bytes_to_buffer(self, ptr: int, data: bytes, length: int) -> None: ...
    def read_bytes_from_buffer(self, ptr: int, length: int) -> bytes: ...
    def transfer_sync_read(self, remote_url: str, dst_ptr: int, src_ptr: int, length: int) -> int: ...
    def register_memory(self, ptr: int, length: int) -> int: ...
    def unregister_memory(self, ptr: int) -> int: ...


def engine_port(stage_idx: int, replica_idx: int) -> int:
    """Fixed engine port so a restarted stage comes back at the same URL:
    ``CONNEX_RS_PORT``, else ``CONNEX_RS_BASE_PORT`` (default 51000 + 100 *
    replica) + stage."""
    if os.getenv("CONNEX_RS_PORT"):
        return int(os.environ["CONNEX_RS_PORT"])
    base = int(os.getenv("CONNEX_RS_BASE_PORT") or 51000 + 100 * replica_idx)
    return base + stage_idx


def create_cx_engine(stage_idx: int, replica_idx: int, model: str, listen_ip: str = "0.0.0.0",
                     advertise_ip: str = "", port: Optional[int] = None, log: Optional[logging.Logger] = None,
                     engine_cls=None):
    """Start the native engine (heartbeat ``CONNEX_RS_HEARTBEAT_MS`` / ``_TIMEOUT_MS``,
    default 1000 / 3000, timeout clamped to >= 1000); -> (engine, url)."""
    log = log or logging.getLogger("connex.pp")
    if engine_cls is None:
        from connex_b200.engine import Engine as engine_cls
    hb = int(os.getenv("CONNEX_RS_HEARTBEAT_MS", "1000"))
    hb_to = int(os.getenv("CONNEX_RS_HEARTBEAT_TIMEOUT_MS", "3000"))
    if hb and hb_to < 1000:
        log.warning("heartbeat timeout %s ms < 1000 gives false failures under load; using 1000", hb_to)
        hb_to = 1000
    eng = engine_cls(model, stage_idx, 0, replica_idx, listen_ip=listen_ip,
                     port=engine_port(stage_idx, replica_idx) if port is None else port,
                     advertise_ip=advertise_ip, heartbeat_ms=hb, heartbeat_timeout_ms=hb_to,
                     spin_us=int(os.getenv("CONNEX_RS_SPIN_US", "500")))
    log.info("stage %s: engine at %s (heartbeat %s/%s ms)", stage_idx, eng.local_url, hb, hb_to)
    return eng, eng.local_url


def verify_engine(engine) -> bool:
    """A started engine answers the surface the endpoint needs."""
    need = ("register_memory", "unregister_memory", "transfer_sync_read", "allocate_managed_buffer")
    return all(hasattr(engine, n) for n in need)
