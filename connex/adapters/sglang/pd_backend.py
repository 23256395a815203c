"""Connex KV transfer backend for SGLang prefill-decode disaggregation.

    python -m sglang.launch_server ... --disaggregation-mode prefill \\
        --disaggregation-transfer-backend connex

SGLang's PD protocol (bootstrap server, decode pre-allocation, chunked sends
from prefill to decode, aux data with the first token, aborts) stays exactly
SGLang's Mooncake backend: the manager *is* ``MooncakeKVManager`` with its
transfer engine replaced by :class:`ConnexTransferEngine` (reference
``connex/adapters/sglang/pd_backend.py:45-183``).  What changes is the data
plane under the engine's ``batch_transfer_sync`` (prefill pushes its KV pages
into the decode instance's pre-allocated pages):

* **inside one NVLink box** (the B200 path): the decode side's KV regions are
  exported as CUDA IPC handles in a per-session record on this host's
  ``/dev/shm``; the prefill side maps them once and moves a whole batch of
  pages with ONE ``copy_segments`` kernel launch (SM stores into the peer's
  HBM over NVLink, bounded waits, status word) instead of one RMA per page;
* **otherwise**: the native engine (``connex_b200.engine.Engine``) posts every
  write with ``put_async`` and waits for them together; a dead peer fails the
  writes within the engine's heartbeat timeout and a restarted instance is
  reconnected under the same identity.

Instances can also register in the front-router PD pools
(``CONNEX_PD_FRONT_ROUTER``, ``CONNEX_PD_HTTP_URL``, ``CONNEX_PD_REPLICA``),
so ``connex.serving.pd_router --engine sglang`` follows scale up and down.

Activation needs no SGLang change: the ``sglang.srt.plugins`` entry point
``connex`` calls :func:`register`, which adds ``connex`` to
``--disaggregation-transfer-backend``, a ``CONNEX`` member to the closed
``TransferBackend`` enum, and routes ``get_kv_class`` to the classes here.
"""
from __future__ import annotations

import json
import logging
import os
import socket
import sys
import threading
from typing import List, Optional

log = logging.getLogger("connex.pd.sglang")

BACKEND = "connex"
PEER_FAILED, TIMEOUT, INVALID = -2, -3, -4


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("", 0))
        return s.getsockname()[1]


def _record_path(session_id: str, shm_dir: str = "/dev/shm") -> str:
    return os.path.join(shm_dir, "connex-sglpd-" + session_id.replace(":", "_").replace("/", "_") + ".json")


def _pid_alive(pid: int) -> bool:
    try:
        os.kill(pid, 0)
        return True
    except ProcessLookupError:
        return False
    except PermissionError:
        return True


class _NvlinkPeers:
    """GPU KV regions of the same-host peers, mapped through CUDA IPC, and
    the one-launch copy into them."""

    def __init__(self, device: int, shm_dir: str):
        import torch
        from connex_b200.parallel.peer import PeerMapper
        self.device = device
        self.shm_dir = shm_dir
        self.mapper = PeerMapper(device)
        self.stream = torch.cuda.Stream(device=device)
        self.peers: dict = {}          # session id -> [(remote base, len, local address)]
        self.lock = threading.Lock()

    def _load(self, session_id: str):
        from connex_b200.parallel.peer import PeerHandle
        try:
            with open(_record_path(session_id, self.shm_dir)) as f:
                rec = json.load(f)
        except (OSError, ValueError):
            return None
        if not _pid_alive(int(rec["pid"])):
            return None
        out = []
        for r in rec["regions"]:
            if int(rec["pid"]) == os.getpid():
                local = r["base"]
            else:
                local = self.mapper.open(PeerHandle(bytes.fromhex(r["handle"]), int(r["offset"]), int(r["len"]),
                                                    int(rec["device"]), int(rec["pid"])))
            out.append((r["base"], r["len"], local))
        return out

    def translate(self, session_id: str, addrs: List[int], lengths: List[int]) -> Optional[List[int]]:
        """Local addresses of the peer ranges, or None when any is not a
        mapped region of that peer (re-reads the record once on a miss)."""
        for attempt in range(2):
            with self.lock:
                regions = self.peers.get(session_id)
                if regions is None or attempt == 1:
                    regions = self._load(session_id)
                    if regions is None:
                        return None
                    self.peers[session_id] = regions
            out = []
            for a, n in zip(addrs, lengths):
                hit = next((loc + (a - b) for b, ln, loc in regions if b <= a and a + n <= b + ln), None)
                if hit is None:
                    break
                out.append(hit)
            else:
                return out
        return None

    def copy(self, srcs: List[int], dsts: List[int], lengths: List[int]) -> int:
        import torch
        from connex_b200 import ops
        segs = [(s, d, n) for s, d, n in zip(srcs, dsts, lengths) if n > 0]
        if not segs:
            return 0
        dev = torch.device("cuda", self.device)
        with torch.cuda.device(dev), torch.cuda.stream(self.stream):
            st = ops.new_status(dev)
            t = torch.tensor(segs, dtype=torch.int64).pin_memory().to(dev, non_blocking=True)
            ops.copy_segments(t, sum(n for *_, n in segs), status=st)
            self.stream.synchronize()
            code = int(st.item())
        return 0 if code == 0 else PEER_FAILED

    def close(self) -> None:
        self.mapper.close()


class ConnexTransferEngine:
    """The transfer-engine surface SGLang's Mooncake KV manager calls.
    Session id = ``host:port`` of the native engine; the peer identity is
    rebuilt from it as ``(sglang-pd, 1001, 0, port)`` (decode endpoints:
    prefill pushes to decode)."""

    def __init__(self, hostname: str, role: str, gpu_id: int = 0, engine_cls=None, timeout_ms: int = 30000,
                 shm_dir: str = "/dev/shm"):
        if engine_cls is None:
            from connex_b200.engine import Engine as engine_cls
        from connex.pd.membership import PD_STAGE
        base = int(os.getenv("CONNEX_RS_PORT", "0"))
        port = base + gpu_id if base else _free_port()
        self.role_stage = PD_STAGE.get(role, 1001)
        self.engine = engine_cls("sglang-pd", self.role_stage, 0, port, listen_ip=hostname, port=port,
                                 heartbeat_ms=int(os.getenv("CONNEX_RS_HEARTBEAT_MS", "1000")),
                                 heartbeat_timeout_ms=int(os.getenv("CONNEX_RS_HEARTBEAT_TIMEOUT_MS", "3000")))
        self.url = self.engine.local_url
        self.session_id = self.url.split("#", 1)[0]
        self.hostname, self.gpu_id, self.timeout_ms = hostname, gpu_id, timeout_ms
        self.shm_dir = shm_dir
        self.device_regions: List[tuple] = []       # (ptr, len) of registered GPU memory
        self._nvl: Optional[_NvlinkPeers] = None
        self._lock = threading.Lock()
        self.stats = {"nvlink_batches": 0, "nvlink_bytes": 0, "engine_writes": 0}
        log.info("connex transfer engine %s (%s)", self.session_id, role)

    # ---- memory -----------------------------------------------------------------
    def _is_device(self, ptr: int) -> bool:
        from connex.pd.dataplane import is_device_ptr
        return is_device_ptr(ptr)

    def _on_device(self, ptr: int) -> bool:
        return any(s <= ptr < s + n for s, n in self.device_regions)

    def _publish(self) -> None:
        """Write this session's GPU regions (IPC handles) for same-host peers."""
        from connex_b200 import ops
        regions = []
        for ptr, n in self.device_regions:
            h, off = ops.ipc_export(ptr, self.gpu_id)
            regions.append({"base": ptr, "len": n, "handle": bytes(h).hex(), "offset": off})
        path = _record_path(self.session_id, self.shm_dir)
        with open(path + ".tmp", "w") as f:
            json.dump({"pid": os.getpid(), "device": self.gpu_id, "regions": regions}, f)
        os.replace(path + ".tmp", path)

    def _add(self, ptr: int, length: int) -> bool:
        if not self._is_device(ptr):
            return False
        self.device_regions.append((ptr, length))
        return True

    def register(self, ptr, length) -> None:
        dev = self._add(ptr, length)
        rc = self.engine.register_memory(ptr, length)
        if rc != 0:
            raise RuntimeError(f"memory registration failed (ret={rc})")
        if dev:
            self._publish()

    def deregister(self, ptr) -> None:
        self.engine.unregister_memory(ptr)
        n = len(self.device_regions)
        self.device_regions = [r for r in self.device_regions if r[0] != ptr]
        if len(self.device_regions) != n:
            self._publish()

    def batch_register(self, ptrs: List[int], lengths: List[int]) -> int:
        rc, dev = 0, False
        for p, n in zip(ptrs, lengths):
            dev = self._add(p, n) or dev
            rc = self.engine.register_memory(p, n) or rc
        if dev:
            self._publish()
        return rc

    def batch_deregister(self, ptrs: List[int]) -> int:
        rc = 0
        for p in ptrs:
            rc = self.engine.unregister_memory(p) or rc
        drop = set(ptrs)
        n = len(self.device_regions)
        self.device_regions = [r for r in self.device_regions if r[0] not in drop]
        if len(self.device_regions) != n:
            self._publish()
        return rc

    # ---- transfers: prefill writes into decode memory ----------------------------
    @staticmethod
    def peer_url(session_id: str, stage: int = 1001) -> str:
        if "#" in session_id:
            return session_id
        return f"{session_id}#sglang-pd|{stage}|0|{session_id.rsplit(':', 1)[1]}"

    def _nvlink(self) -> Optional[_NvlinkPeers]:
        import torch
        if not torch.cuda.is_available():
            return None
        if self._nvl is None and self.device_regions:
            with self._lock:
                if self._nvl is None:
                    self._nvl = _NvlinkPeers(self.gpu_id, self.shm_dir)
        return self._nvl

    def transfer_sync(self, session_id: str, buffer: int, peer_buffer_address: int, length: int) -> int:
        return self.batch_transfer_sync(session_id, [buffer], [peer_buffer_address], [length])

    def batch_transfer_sync(self, session_id: str, buffers: List[int], peer_buffer_addresses: List[int],
                            lengths: List[int]) -> int:
        """0, or PEER_FAILED (-2) / TIMEOUT (-3) / INVALID (-4)."""
        if not buffers:
            return 0
        on_dev = [self._on_device(b) for b in buffers]
        if any(on_dev):
            nvl = self._nvlink()
            dsts = nvl.translate(session_id, peer_buffer_addresses, lengths) if nvl is not None else None
            if dsts is None or not all(on_dev):
                # GPU pages need the NVLink route (the native engine moves host memory)
                log.error("no NVLink route from %s to the KV of %s", self.session_id, session_id)
                return INVALID
            rc = nvl.copy(buffers, dsts, lengths)
            self.stats["nvlink_batches"] += 1
            self.stats["nvlink_bytes"] += sum(lengths)
            return rc
        return self._engine_writes(session_id, buffers, peer_buffer_addresses, lengths)

    def _engine_writes(self, session_id, buffers, peer_addrs, lengths) -> int:
        url = self.peer_url(session_id)
        put = getattr(self.engine, "put_async", None)
        if put is None:
            for b, p, n in zip(buffers, peer_addrs, lengths):
                rc = self.engine.transfer_sync_write(url, b, p, n, self.timeout_ms)
                if rc < 0:
                    return rc
            return 0
        handles, rc = [], 0
        try:
            for b, p, n in zip(buffers, peer_addrs, lengths):
                handles.append(put(url, b, p, n, self.timeout_ms))
        except Exception as ex:  # noqa: BLE001
            log.warning("posting writes to %s failed: %s", session_id, ex)
            rc = PEER_FAILED
        for h in handles:                   # drain everything posted before reporting
            try:
                if not h.wait(self.timeout_ms + 1000):
                    rc = rc or TIMEOUT
            except Exception:  # noqa: BLE001
                rc = rc or PEER_FAILED
        self.stats["engine_writes"] += len(handles)
        if rc:
            log.warning("%d writes to %s failed (rc=%d)", len(handles), session_id, rc)
        return rc

    # ---- misc ----------------------------------------------------------------------
    def get_session_id(self) -> str:
        return self.session_id

    def send_probe(self, peer_session_id: str) -> int:
        try:
            self.engine.connect(self.peer_url(peer_session_id))
            return 0
        except Exception:  # noqa: BLE001
            return -1

    def get_engine(self):
        return self.engine

    def get_ib_device(self) -> str:
        return os.getenv("UCX_NET_DEVICES", "")

    def close(self) -> None:
        try:
            os.unlink(_record_path(self.session_id, self.shm_dir))
        except OSError:
            pass
        if self._nvl is not None:
            self._nvl.close()


ConnexRsTransferEngine = ConnexTransferEngine     # the reference's class name

_ENGINE: Optional[ConnexTransferEngine] = None
_ENGINE_LOCK = threading.Lock()
_MEMBER = None
_REPORTER = None


def get_engine(hostname: str, role: str, gpu_id: int) -> ConnexTransferEngine:
    """One transfer engine per process (SGLang builds one manager per rank)."""
    global _ENGINE
    with _ENGINE_LOCK:
        if _ENGINE is None:
            _ENGINE = ConnexTransferEngine(hostname, role, gpu_id)
        return _ENGINE


def _maybe_register_member(role: str, rank: int, tp_size: int = 1, engine=None) -> None:
    """Register this TP rank in the front-router PD pools as shard ``rank`` of
    a group of ``tp_size`` (listed only while every rank holds its lease)."""
    global _MEMBER, _REPORTER
    fr, url = os.getenv("CONNEX_PD_FRONT_ROUTER"), os.getenv("CONNEX_PD_HTTP_URL")
    if not fr or not url or _MEMBER is not None:
        return
    from connex.pd.membership import PDMember
    model = os.getenv("CONNEX_PD_MODEL", "default")
    extra = [f"rs={engine.session_id}"] if engine is not None else []
    _MEMBER = PDMember(fr, model, role, int(os.getenv("CONNEX_PD_REPLICA", "0")), url,
                       kv_addr=os.getenv("CONNEX_PD_BOOTSTRAP") if role == "prefill" else None,
                       shard=rank, group_size=max(1, tp_size), extra_addresses=extra)
    _MEMBER.start()
    if engine is not None and hasattr(engine.engine, "wait_event"):
        # a peer rank's death (engine event) fails its whole group at once
        from connex.pd.group import PeerDeathReporter, rs_port_resolver
        _REPORTER = PeerDeathReporter(engine.engine, fr, "sglang-pd", resolve=rs_port_resolver(fr, model))
        _REPORTER.start()


def _classes():
    """The backend classes (SGLang imported lazily)."""
    from sglang.srt.disaggregation.mooncake.conn import (MooncakeKVBootstrapServer, MooncakeKVManager,
                                                         MooncakeKVReceiver, MooncakeKVSender)
    from sglang.srt.disaggregation.utils import DisaggregationMode

    class ConnexKVManager(MooncakeKVManager):
        def init_engine(self):
            role = "prefill" if self.disaggregation_mode == DisaggregationMode.PREFILL else "decode"
            self.engine = get_engine(self.local_ip, role, int(self.kv_args.gpu_id))
            try:
                tp = int(getattr(self, "attn_tp_size", 1) or 1)
                _maybe_register_member(role, int(self.kv_args.engine_rank) % tp, tp, engine=self.engine)
            except Exception as ex:  # noqa: BLE001  membership is optional
                log.warning("front-router registration failed: %s", ex)

    class ConnexKVSender(MooncakeKVSender):
        pass

    class ConnexKVReceiver(MooncakeKVReceiver):
        pass

    class ConnexKVBootstrapServer(MooncakeKVBootstrapServer):
        pass

    return ConnexKVManager, ConnexKVSender, ConnexKVReceiver, ConnexKVBootstrapServer


def extend_enum(enum_cls, name: str, value):
    """Add member ``name = value`` to an existing Enum class (idempotent)."""
    hit = enum_cls._value2member_map_.get(value)
    if hit is not None:
        return hit
    base = getattr(enum_cls, "_member_type_", object)
    member = object.__new__(enum_cls) if base is object else base.__new__(enum_cls, value)
    member._name_, member._value_ = name, value
    member.__objclass__ = enum_cls
    if hasattr(next(iter(enum_cls), None), "_sort_order_"):
        member._sort_order_ = len(enum_cls._member_names_)
    enum_cls._member_map_[name] = member
    enum_cls._value2member_map_[value] = member
    enum_cls._member_names_.append(name)
    type.__setattr__(enum_cls, name, member)
    return member


_extend_enum = extend_enum


def _native_backend() -> bool:
    """This SGLang ships a ``connex`` backend itself."""
    import importlib.util
    try:
        return importlib.util.find_spec("sglang.srt.disaggregation.connex") is not None
    except ImportError:
        return False


def _allow_staging_buffer() -> None:
    """Heterogeneous attention TP between prefill and decode needs SGLang's
    staging buffer (``SGLANG_DISAGG_STAGING_BUFFER=1``); SGLang's argument
    check names only its own backends, so let ``connex`` through it."""
    try:
        import sglang.srt.arg_groups.pd_disaggregation_hook as hook
        from sglang.srt.environ import envs
    except ImportError:
        return
    check0 = hook.handle_pd_disaggregation
    if getattr(check0, "_connex", False):
        return

    def handle_pd_disaggregation(server_args):
        flag = envs.SGLANG_DISAGG_STAGING_BUFFER
        if getattr(server_args, "disaggregation_transfer_backend", None) != BACKEND or not flag.get():
            return check0(server_args)
        get0 = flag.get
        flag.get = lambda *a, **k: False           # only around the backend-name check
        try:
            return check0(server_args)
        finally:
            flag.get = get0

    handle_pd_disaggregation._connex = True
    hook.handle_pd_disaggregation = handle_pd_disaggregation


def register() -> None:
    """``sglang.srt.plugins`` entry point: make ``connex`` a transfer backend."""
    import sglang.srt.disaggregation.utils as du
    if BACKEND in du.TransferBackend._value2member_map_ and not getattr(du.get_kv_class, "_connex", False) \
            and _native_backend():
        return
    try:
        from sglang.srt.arg_groups.choices import (DISAGG_TRANSFER_BACKEND_CHOICES,
                                                   add_disagg_transfer_backend_choices)
        if BACKEND not in DISAGG_TRANSFER_BACKEND_CHOICES:
            add_disagg_transfer_backend_choices([BACKEND])
    except ImportError:
        log.warning("could not extend --disaggregation-transfer-backend choices")
    _allow_staging_buffer()
    member = extend_enum(du.TransferBackend, "CONNEX", BACKEND)
    if getattr(du.get_kv_class, "_connex", False):
        return
    lookup0 = du.get_kv_class

    def get_kv_class(transfer_backend, class_type):
        if transfer_backend is member or getattr(transfer_backend, "value", None) == BACKEND:
            if class_type == du.KVClassType.KVARGS:
                from sglang.srt.disaggregation.base import KVArgs
                return KVArgs
            mgr, snd, rcv, boot = _classes()
            return {du.KVClassType.MANAGER: mgr, du.KVClassType.SENDER: snd, du.KVClassType.RECEIVER: rcv,
                    du.KVClassType.BOOTSTRAP_SERVER: boot}.get(class_type)
        return lookup0(transfer_backend, class_type)

    get_kv_class._connex = True
    du.get_kv_class = get_kv_class
    for mod in list(sys.modules.values()):          # modules that imported the name before us
        if mod is not None and getattr(mod, "get_kv_class", None) is lookup0:
            mod.get_kv_class = get_kv_class
    log.info("SGLang transfer backend %r registered", BACKEND)


__all__ = ["ConnexTransferEngine", "ConnexRsTransferEngine", "get_engine", "register", "extend_enum", "BACKEND"]
