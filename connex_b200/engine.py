"""Python face of the native transfer engine (``connex_b200._cxengine``).

:class:`Engine` has the surface of a one-sided transfer engine: identity
``(model, stage, shard, replica)``, ``local_url = "ip:port#model|stage|shard|replica"``,
managed / registered memory, ``transfer_sync_read/write``, ``get_async`` /
``put_async`` / ``put_signal`` handles, messages, peer events
(``up`` / ``joined`` / ``failed``) and counters.  Error codes:
``PEER_FAILED`` (-2), ``TIMEOUT`` (-3), ``INVALID`` (-4), ``CANCELLED`` (-5).

Device memory: ``allocate_device_buffer(size, device)`` gives a GPU range
(a VMM allocation) that peers on the same machine map and reach with the
copy engines; any other registered device range (a torch tensor) is exported
through its legacy IPC handle.  Device ranges are never served over the
socket path (a peer on another machine gets ``INVALID``).  ``put_chain`` is
the doorbell -> gate -> payload -> flag chain of a ring channel.  A dead
peer's mappings are released once the copies that touched them have passed
(``reap``; also run by the heartbeat thread).  :class:`DeviceBuffer` /
:class:`Mapping` are the same export / import for buffers shared without an
engine (:mod:`connex_b200.parallel.peer`).

:class:`CxEngineTransport` adapts it to the ``ElasticPeerSet`` transport duck
type, and :func:`url_identity` parses identities out of engine URLs.
"""
from __future__ import annotations

from typing import Any, Optional, Tuple

from connex_b200._cxengine import (CANCELLED, INVALID, OK, PEER_FAILED, TIMEOUT, DeviceBuffer, Engine,  # noqa: F401
                                   Handle, Mapping, boot_id, device_memory_info, device_plane)


def url_identity(url: str) -> Optional[Tuple[str, int, int, int]]:
    """``"ip:port#model|stage|shard|replica"`` -> identity tuple (None without one)."""
    if "#" not in url:
        return None
    m, s, sh, r = url.split("#", 1)[1].split("|")
    return m, int(s), int(sh), int(r)


def url_hostport(url: str) -> str:
    return url.split("#", 1)[0]


class CxEngineTransport:
    """``connect_sync / send_sync / close_endpoint`` over engine messages."""

    def __init__(self, engine: Engine):
        self.engine = engine

    def connect_sync(self, host: str, port: int) -> Any:
        url = f"{host}:{port}"
        if not self.engine.connect(url):
            raise ConnectionError(f"cannot reach {url}")
        return url

    def send_sync(self, ep: Any, data: bytes, tag: int = 0) -> None:
        if not self.engine.send_msg(ep, bytes(data)):
            raise ConnectionError(f"send to {ep} failed")

    def recv_sync(self, timeout_ms: int = 1000):
        m = self.engine.recv_msg(timeout_ms)
        return None if m is None else m[1]

    def close_endpoint(self, ep: Any) -> bool:
        return True

    def stop_sync(self) -> None:
        self.engine.close()
