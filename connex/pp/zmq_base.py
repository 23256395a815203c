"""ZeroMQ stage sockets and the ZeroMQ-only tensor-dict path (reference
``connex/pp/zmq_base.py:42-389``).

One ROUTER per stage (bound at ``router_port``; receives forward steps and
returns) and DEALERs to peers.  The ZeroMQ-only wire, kept byte-compatible
with the reference so mixed deployments interoperate, is one multi-frame
message per dict::

    [!Q len(meta), meta = pickle({"metadata_list", "send_timestamp"}), !Q n]
    + n x [!Q len(t), torch.save(t.cpu())]

``metadata_list`` = ``[(key, TensorMetadata(device, dtype, size)) | (key, value)]``;
:class:`TensorDictCodec` is injectable so an engine can plug in its own
metadata class.  The optional control socket speaks the legacy front-ROUTER
``REGISTER`` / ``ASSIGN`` JSON.
"""
from __future__ import annotations

import io
import json
import logging
import pickle
import struct
import time
from collections import namedtuple
from typing import Any, List, Optional, Tuple
from uuid import uuid4

import zmq

from connex.pp.hooks import NULL_METRICS, NetUtils

TensorMetadata = namedtuple("TensorMetadata", ["device", "dtype", "size"])
_LEN = struct.Struct("!Q")


class TensorDictCodec:
    """(metadata_list, tensors) <-> tensor dict."""

    def __init__(self, meta_cls=TensorMetadata, split=None):
        self.meta_cls = meta_cls
        self._split = split

    def split(self, td: dict):
        if self._split is not None:
            return self._split(td)
        import torch
        meta, tensors = [], []
        for k, v in td.items():
            if isinstance(v, torch.Tensor):
                meta.append((k, self.meta_cls(v.device.type, v.dtype, v.size())))
                tensors.append(v)
            else:
                meta.append((k, v))
        return meta, tensors

    def is_tensor_meta(self, v) -> bool:
        return isinstance(v, self.meta_cls)


DEFAULT_CODEC = TensorDictCodec()


def encode_frames(td: dict, codec: TensorDictCodec = DEFAULT_CODEC, send_ts: Optional[float] = None) -> List[bytes]:
    import torch
    meta, tensors = codec.split(td)
    mb = pickle.dumps({"metadata_list": meta, "send_timestamp": time.time() if send_ts is None else send_ts})
    frames = [_LEN.pack(len(mb)), mb, _LEN.pack(len(tensors))]
    for t in tensors:
        buf = io.BytesIO()
        torch.save(t.detach().cpu(), buf)
        b = buf.getvalue()
        frames += [_LEN.pack(len(b)), b]
    return frames


def decode_frames(frames: List[bytes], device: str = "cpu", codec: TensorDictCodec = DEFAULT_CODEC):
    """-> (tensor dict, send_timestamp)."""
    import torch
    meta = pickle.loads(frames[1])
    n = _LEN.unpack(frames[2])[0]
    tensors = [torch.load(io.BytesIO(frames[3 + 2 * i + 1]), weights_only=True) for i in range(n)]
    out, it = {}, iter(tensors)
    for k, v in meta["metadata_list"]:
        if codec.is_tensor_meta(v):
            t = next(it)
            out[k] = t.to(device) if device != "cpu" else t
        else:
            out[k] = v
    return out, meta.get("send_timestamp")


class ZmqStageBase:
    """ROUTER/DEALER stage endpoint with the ZeroMQ-only data path.

    Stage 0 sends forward over a DEALER to stage 1's ROUTER; every later
    stage receives on its ROUTER and forwards to the next; the last stage
    returns to stage 0's ROUTER.  Peers come from ``assign`` (legacy control
    socket) or are set with :meth:`set_peers`."""

    log: logging.Logger = logging.getLogger("connex.pp")
    net = NetUtils
    codec: TensorDictCodec = DEFAULT_CODEC
    metrics = NULL_METRICS
    backend_name = "zmq"

    def __init__(self, stage_idx: int, num_stages: int, router_port: int = 0, front_router_addr: Optional[str] = None,
                 device: str = "cpu", timeout_ms: int = -1, host: Optional[str] = None):
        self.stage_idx, self.num_stages = stage_idx, num_stages
        self.is_first, self.is_last = stage_idx == 0, stage_idx == num_stages - 1
        self.device = device
        self.timeout_ms = timeout_ms
        self.ctx = zmq.Context()
        self.router = self.ctx.socket(zmq.ROUTER)
        self.router.setsockopt(zmq.LINGER, 0)
        ip = host or self.net.get_ip()
        if router_port:
            self.router.bind(f"tcp://{ip}:{router_port}")
        else:
            router_port = self.router.bind_to_random_port(f"tcp://{ip}")
        self.router_port = router_port
        self.router_endpoint = self.net.get_tcp_uri(ip, router_port)
        self.forward_socket: Optional[zmq.Socket] = None
        self.return_socket: Optional[zmq.Socket] = None
        self.front_router_addr = front_router_addr
        self.control: Optional[zmq.Socket] = None
        self._last_sender: Optional[bytes] = None

    def _dealer(self, addr: str) -> zmq.Socket:
        s = self.ctx.socket(zmq.DEALER)
        s.setsockopt(zmq.LINGER, 0)
        s.setsockopt(zmq.IDENTITY, f"cx-{self.stage_idx}-{uuid4().hex[:8]}".encode())
        s.connect(addr)
        return s

    def set_peers(self, forward: Optional[str] = None, head: Optional[str] = None) -> None:
        """``forward``: next stage's ROUTER; ``head``: stage 0's ROUTER (last stage)."""
        for s in (self.forward_socket, self.return_socket):
            if s is not None:
                s.close(0)
        self.forward_socket = self._dealer(forward) if forward else None
        self.return_socket = self._dealer(head) if head else None

    # legacy control plane: REGISTER -> ASSIGN {"forward", "head"}
    def register(self, model: str = "default", replica_idx: int = 0, timeout_ms: int = 2000) -> bool:
        if not self.front_router_addr:
            return False
        self.control = self.ctx.socket(zmq.DEALER)
        self.control.setsockopt(zmq.LINGER, 0)
        self.control.connect(self.front_router_addr)
        self.control.send(json.dumps({"type": "REGISTER", "stage": self.stage_idx, "replica": replica_idx,
                                      "model": model, "endpoint": self.router_endpoint}).encode())
        if not self.control.poll(timeout_ms):
            return False
        msg = json.loads(self.control.recv())
        if msg.get("type") == "ASSIGN":
            self.set_peers(msg.get("forward"), msg.get("head"))
            return True
        return False

    def send_tensor_dict(self, td: dict) -> None:
        sock = self.return_socket if self.is_last else self.forward_socket
        if sock is None:
            raise RuntimeError(f"stage {self.stage_idx}: no peer to send to")
        frames = encode_frames(td, self.codec)
        sock.send_multipart(frames, copy=False)
        self.metrics.inc("bytes_sent", float(sum(len(f) for f in frames)))

    def recv_tensor_dict(self, timeout_ms: Optional[int] = None) -> Optional[dict]:
        t = self.timeout_ms if timeout_ms is None else timeout_ms
        if t is not None and t >= 0 and not self.router.poll(t):
            return None
        frames = self.router.recv_multipart()
        self._last_sender = frames[0]
        td, ts = decode_frames(frames[1:], self.device, self.codec)
        if ts:
            self.metrics.observe("transfer_latency", max(0.0, time.time() - ts))
        return td

    def close(self) -> None:
        for s in (self.forward_socket, self.return_socket, self.control, self.router):
            if s is not None:
                s.close(0)
        self.ctx.term()
