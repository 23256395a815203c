"""Weight sync for SGLang through its custom weight-loader hook.

Start the server with ``--custom-weight-loader connex.rl.sglang_ext.connex_load``
and call its ``update_weights_from_tensor`` route with ``load_format`` =
:data:`LOADER` and the single control tensor of :func:`control_payload` (a
JSON record as bytes: registry URL, version, member name, transport, chunk
size).  Every TP scheduler process then runs :func:`connex_load`: it keeps
one :class:`connex.rl.sync.WeightSubscriber` per process, pulls the named
version through the weight-sync transport and hands the tensors to the
model's ``load_weights``.  A call without the control tensor loads the given
tensors as usual.

Interface parity: ``connex/rl/sglang_ext.py:36-87`` of the reference (the
loader name, the control tensor name and record keys are the contract).
"""
from __future__ import annotations

import json
import os
import socket
from typing import Optional

import torch

from .registry import RegistryClient
from .sync import DEFAULT_CHUNK, WeightSubscriber
from .transport import make_transport

LOADER = "connex.rl.sglang_ext.connex_load"
CONTROL = "__connex_weight_sync__"

_SUBSCRIBER: Optional[WeightSubscriber] = None
last_stats: dict = {}


def control_payload(registry_url, version=None, member=None, transport="engine", chunk_bytes=DEFAULT_CHUNK):
    record = json.dumps({"registry_url": registry_url, "version": version, "member": member,
                         "transport": transport, "chunk_bytes": chunk_bytes}).encode()
    return [(CONTROL, torch.frombuffer(bytearray(record), dtype=torch.uint8))]


def parse_control(named_tensors):
    """The control record among ``named_tensors``, or None."""
    found = [t for name, t in named_tensors if name == CONTROL]
    if not found:
        return None
    return json.loads(bytes(found[0].cpu().tolist()).decode())


def _tp_rank() -> int:
    env = os.environ.get("CONNEX_TP_RANK")
    if env is not None:
        return int(env)
    return torch.cuda.current_device() if torch.cuda.is_available() else 0


def _load_device() -> torch.device:
    if os.environ.get("CONNEX_RL_DEVICE"):
        return torch.device(os.environ["CONNEX_RL_DEVICE"])
    if torch.cuda.is_available():
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def _subscriber(ctl: dict, device) -> WeightSubscriber:
    """This process's subscriber, created on the first update."""
    global _SUBSCRIBER
    if _SUBSCRIBER is None:
        rank = _tp_rank()
        member = f"{ctl.get('member') or f'{socket.gethostname()}-{os.getpid()}'}/r{rank}"
        kind = ctl.get("transport") or "engine"
        if kind in ("local", "nvlink"):
            transport = make_transport(kind, name=member)
        else:
            transport = make_transport(kind, lid=("connex-rl", 1, rank, os.getpid()))
        _SUBSCRIBER = WeightSubscriber(RegistryClient(ctl["registry_url"]), transport, member, device=device,
                                       chunk_bytes=ctl.get("chunk_bytes", DEFAULT_CHUNK),
                                       arena="host" if kind == "engine" else "device")
    return _SUBSCRIBER


def reset_subscriber(leave: bool = True) -> None:
    """Close this process's subscriber (the next update creates a new one)."""
    global _SUBSCRIBER
    if _SUBSCRIBER is not None:
        _SUBSCRIBER.close(leave=leave)
        _SUBSCRIBER = None


def connex_load(model, named_tensors):
    """SGLang custom weight loader (see the module docstring)."""
    global last_stats
    named_tensors = list(named_tensors)
    ctl = parse_control(named_tensors)
    if ctl is None:
        model.load_weights(named_tensors)
        return
    device = _load_device()
    sub = _subscriber(ctl, device)
    manifest = sub.pull(ctl.get("version"))
    model.load_weights(list(sub.tensors()))
    if device.type == "cuda":
        torch.cuda.current_stream(device).synchronize()
    sub.commit(manifest.version)
    last_stats = dict(sub.stats)
