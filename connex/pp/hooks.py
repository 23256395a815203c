"""Engine-facing protocols of the pipeline step protocol, metrics sinks and
network helpers (reference ``connex/pp/hooks.py:31-223``).

* :class:`EngineHooks` -- what an engine provides: ``kv_held`` / ``release``
  (stages 1..), ``reprefill`` / ``abort`` (stage 0).
* :class:`StepTransport` -- the step-level API of a pipeline endpoint that
  :mod:`connex.pp.link` drives.
* :class:`MetricsSink` with :data:`METRIC_NAMES`, :class:`NullMetrics` and
  :class:`PrefixedPrometheusSink`.
"""
from __future__ import annotations

import ipaddress
import logging
import os
import socket
from typing import Any, Iterable, Optional, Protocol, Sequence, runtime_checkable


# ---- network helpers ------------------------------------------------------------
def _is_ipv6(host: str) -> bool:
    try:
        return isinstance(ipaddress.ip_address(host), ipaddress.IPv6Address)
    except ValueError:
        return False


def get_ip() -> str:
    """This host's address: ``CONNEX_HOST_IP`` / ``VLLM_HOST_IP`` or the
    interface of the default route (a UDP connect sends no packet)."""
    env = os.getenv("CONNEX_HOST_IP") or os.getenv("VLLM_HOST_IP")
    if env:
        return env
    for fam, probe in ((socket.AF_INET, ("8.8.8.8", 80)), (socket.AF_INET6, ("2001:4860:4860::8888", 80))):
        try:
            with socket.socket(fam, socket.SOCK_DGRAM) as s:
                s.connect(probe)
                return s.getsockname()[0]
        except OSError:
            pass
    logging.getLogger("connex.pp").warning("no routable address found; using 0.0.0.0 (set CONNEX_HOST_IP)")
    return "0.0.0.0"


def get_tcp_uri(ip: str, port: int) -> str:
    return f"tcp://[{ip}]:{port}" if _is_ipv6(ip) else f"tcp://{ip}:{port}"


def join_host_port(host: str, port: int) -> str:
    return f"[{host}]:{port}" if _is_ipv6(host) else f"{host}:{port}"


def split_host_port(host_port: str) -> tuple:
    if host_port.startswith("["):
        host, rest = host_port[1:].split("]", 1)
        return host, int(rest.lstrip(":"))
    host, port = host_port.rsplit(":", 1)
    return host, int(port)


class NetUtils:
    get_ip = staticmethod(get_ip)
    get_tcp_uri = staticmethod(get_tcp_uri)
    join_host_port = staticmethod(join_host_port)
    split_host_port = staticmethod(split_host_port)


# ---- metrics ----------------------------------------------------------------------
METRIC_NAMES = (
    "bytes_sent", "bytes_received", "messages_sent", "messages_received",
    "send_latency", "recv_latency", "enqueue_latency", "delivery_latency",
    "delivery_latency_local", "ready_to_use_latency", "tensor_count", "tensor_size",
    "serialization_latency", "deserialization_latency", "buffer_copy_latency",
    "errors", "connection_status",
    "connection_ready_time", "connection_rdma_setup_time", "connection_ready_timestamp",
    "connection_discovery_time",
)


class MetricsSink(Protocol):
    enabled: bool

    def observe(self, name: str, value: float, **labels: str) -> None: ...

    def inc(self, name: str, value: float = 1.0, **labels: str) -> None: ...

    def set(self, name: str, value: float, **labels: str) -> None: ...


class NullMetrics:
    enabled = False

    def observe(self, name, value, **labels):
        pass

    def inc(self, name, value=1.0, **labels):
        pass

    def set(self, name, value, **labels):
        pass


NULL_METRICS = NullMetrics()


class RecordingMetrics:
    """In-memory sink (tests, local debugging): ``values[name]`` lists observations."""

    enabled = True

    def __init__(self):
        self.values: dict = {}

    def observe(self, name, value, **labels):
        self.values.setdefault(name, []).append((value, labels))

    inc = observe
    set = observe


class PrefixedPrometheusSink:
    """Binds metric names to prometheus collectors ``<prefix>comm_<name>`` (or
    ``<prefix><name>``) of ``module`` with labels backend / stage_idx + the
    call's labels; children are bound once per label set."""

    enabled = True

    def __init__(self, module: Any, prefix: str, backend: str, stage_idx: int):
        self.module, self.prefix = module, prefix
        self.base = {"backend": backend, "stage_idx": stage_idx}
        self._children: dict = {}

    def _child(self, name: str, labels: dict):
        key = (name, tuple(sorted(labels.items())))
        ch = self._children.get(key)
        if ch is None:
            m = getattr(self.module, f"{self.prefix}comm_{name}", None) or \
                getattr(self.module, f"{self.prefix}{name}", None)
            ch = m.labels(**self.base, **labels) if m is not None else False
            self._children[key] = ch
        return ch

    def observe(self, name, value, **labels):
        ch = self._child(name, labels)
        if ch:
            ch.observe(value)

    def inc(self, name, value=1.0, **labels):
        ch = self._child(name, labels)
        if ch:
            ch.inc(value)

    def set(self, name, value, **labels):
        ch = self._child(name, labels)
        if ch:
            ch.set(value)


# ---- engine contract ------------------------------------------------------------
RequestId = Any


@runtime_checkable
class EngineHooks(Protocol):
    def kv_held(self, request_id: RequestId) -> int:
        """Stages 1..: leading tokens of the request whose KV this stage itself
        computed and still holds (a fresh replica after failover holds 0)."""
        ...

    def release(self, request_ids: Iterable[RequestId]) -> None:
        """Drop all per-request state (KV blocks) of these requests."""
        ...

    def reprefill(self, request_ids: Sequence[RequestId]) -> None:
        """Stage 0: discard this step's token for them and recompute them
        (prompt + generated tokens) on the current chain."""
        ...

    def abort(self, request_ids: Sequence[RequestId]) -> None:
        """Stage 0: finish them with an error (re-prefill budget exhausted)."""
        ...


class StepTransport(Protocol):
    stage_idx: int
    num_stages: int
    is_first: bool
    is_last: bool

    @property
    def inflight(self) -> int: ...

    def new_step_id(self) -> int: ...

    def send_step(self, tensor_dict: dict, corr: int, dst: Optional[int] = None) -> None: ...

    def recv_step(self, corr: int, timeout_s: Optional[float] = None) -> Optional[dict]: ...

    def abandon_step(self, corr: int) -> None: ...

    def recv_forward(self) -> tuple: ...

    def send_reply(self, tensor_dict: dict, ctx: Optional[tuple]) -> None: ...

    def downstream_healthy(self) -> bool: ...
