"""What the pipeline step protocol needs from an engine, metrics sinks, and
address helpers.

* :class:`EngineHooks` -- the engine side of the protocol: ``kv_held`` and
  ``release`` on stages 1.., ``reprefill`` and ``abort`` on stage 0.
* :class:`StepTransport` -- the step-level API of a pipeline endpoint that
  :mod:`connex.pp.link` drives (K steps in flight, per-step ids).
* Metrics: the :class:`MetricsSink` protocol and the metric names the PP
  data plane reports (:data:`METRIC_NAMES`), a null sink, an in-memory sink
  and a Prometheus binding (:class:`PrefixedPrometheusSink`).
* Address helpers for IPv4 / IPv6 ``host:port`` strings and ZeroMQ URIs,
  and this host's routable address (``CONNEX_HOST_IP``).

Interface parity: ``connex/pp/hooks.py:31-223`` of the reference (protocol
method names and metric names are part of the public contract).
"""
from __future__ import annotations

import ipaddress
import logging
import os
import socket
from typing import Any, Callable, Dict, Iterable, Optional, Protocol, Sequence, Tuple, runtime_checkable

_log = logging.getLogger("connex.pp")


# ---------------------------------------------------------------- addresses
def _ipv6(host: str) -> bool:
    try:
        return ipaddress.ip_address(host).version == 6
    except ValueError:
        return False


def _bracket(host: str) -> str:
    return f"[{host}]" if _ipv6(host) else host


def get_ip() -> str:
    """This host's address for peers to dial: ``CONNEX_HOST_IP`` (or
    ``VLLM_HOST_IP``) when set, else the source address of the default route
    (found with a connected UDP socket, which sends nothing)."""
    for var in ("CONNEX_HOST_IP", "VLLM_HOST_IP"):
        if os.getenv(var):
            return os.environ[var]
    probes = ((socket.AF_INET, "8.8.8.8"), (socket.AF_INET6, "2001:4860:4860::8888"))
    for family, target in probes:
        try:
            with socket.socket(family, socket.SOCK_DGRAM) as s:
                s.connect((target, 80))
                return s.getsockname()[0]
        except OSError:
            continue
    _log.warning("no routable address found; using 0.0.0.0 (set CONNEX_HOST_IP)")
    return "0.0.0.0"


def get_tcp_uri(ip: str, port: int) -> str:
    return f"tcp://{_bracket(ip)}:{port}"


def join_host_port(host: str, port: int) -> str:
    return f"{_bracket(host)}:{port}"


def split_host_port(host_port: str) -> Tuple[str, int]:
    """``"h:p"`` or ``"[v6]:p"`` -> (host, port)."""
    host, sep, port = host_port.rpartition(":")
    if not sep:
        raise ValueError(f"no port in {host_port!r}")
    return host.strip("[]"), int(port)


class NetUtils:
    """The address helpers as one namespace (injectable in tests)."""

    get_ip = staticmethod(get_ip)
    get_tcp_uri = staticmethod(get_tcp_uri)
    join_host_port = staticmethod(join_host_port)
    split_host_port = staticmethod(split_host_port)


# ------------------------------------------------------------------ metrics
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
    """Discards everything (the default sink)."""

    enabled = False

    def observe(self, name, value, **labels):
        return None

    def inc(self, name, value=1.0, **labels):
        return None

    def set(self, name, value, **labels):
        return None


NULL_METRICS = NullMetrics()


class RecordingMetrics:
    """Keeps every call in memory: ``values[name]`` is a list of
    ``(value, labels)`` in call order (tests, local debugging)."""

    enabled = True

    def __init__(self):
        self.values: Dict[str, list] = {}

    def _record(self, name, value, **labels):
        self.values.setdefault(name, []).append((value, labels))

    def observe(self, name, value, **labels):
        self._record(name, value, **labels)

    def inc(self, name, value=1.0, **labels):
        self._record(name, value, **labels)

    def set(self, name, value, **labels):
        self._record(name, value, **labels)


class PrefixedPrometheusSink:
    """Forwards metric calls to Prometheus collectors that an engine defines
    in ``module`` as ``<prefix>comm_<name>`` (or ``<prefix><name>``), labelled
    with ``backend`` and ``stage_idx`` plus the call's own labels.  A name
    without a collector is ignored.  The labelled child of each (name,
    labels) pair is resolved once and reused."""

    enabled = True

    def __init__(self, module: Any, prefix: str, backend: str, stage_idx: int):
        self.module, self.prefix = module, prefix
        self.base = {"backend": backend, "stage_idx": stage_idx}
        self._bound: Dict[tuple, Any] = {}

    def _collector(self, name: str):
        for attr in (f"{self.prefix}comm_{name}", f"{self.prefix}{name}"):
            c = getattr(self.module, attr, None)
            if c is not None:
                return c
        return None

    def _apply(self, op: str, name: str, value: float, labels: dict) -> None:
        key = (name, frozenset(labels.items()))
        child = self._bound.get(key)
        if child is None:
            coll = self._collector(name)
            child = coll.labels(**self.base, **labels) if coll is not None else False
            self._bound[key] = child
        if child is not False:
            getattr(child, op)(value)

    def observe(self, name, value, **labels):
        self._apply("observe", name, value, labels)

    def inc(self, name, value=1.0, **labels):
        self._apply("inc", name, value, labels)

    def set(self, name, value, **labels):
        self._apply("set", name, value, labels)


# -------------------------------------------------------- engine contract
RequestId = Any


@runtime_checkable
class EngineHooks(Protocol):
    def kv_held(self, request_id: RequestId) -> int:
        """Stages 1..: how many leading tokens of the request this stage has
        computed itself and still holds (0 on a replica new to it)."""
        ...

    def release(self, request_ids: Iterable[RequestId]) -> None:
        """Drop every per-request state (KV blocks) of these requests."""
        ...

    def reprefill(self, request_ids: Sequence[RequestId]) -> None:
        """Stage 0: discard this step's token of each and recompute them
        (prompt plus generated tokens) on the current chain."""
        ...

    def abort(self, request_ids: Sequence[RequestId]) -> None:
        """Stage 0: finish them with an error (re-prefill budget used up)."""
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


MetricsFactory = Callable[[int], MetricsSink]
