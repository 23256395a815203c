"""Weight sync for SGLang through its custom weight-loader hook (reference
``connex/rl/sglang_ext.py:36-87``).

Start the server with ``--custom-weight-loader connex.rl.sglang_ext.connex_load``
and call ``update_weights_from_tensor`` with ``load_format`` = :data:`LOADER`
and the one control tensor from :func:`control_payload`.  Each TP scheduler
process then runs :func:`connex_load`, which pulls the version with one
:class:`WeightSubscriber` per process and calls ``model.load_weights``.
"""
from __future__ import annotations

import json
import os
import socket

import torch

from .registry import RegistryClient
from .sync import DEFAULT_CHUNK, WeightSubscriber
from .transport import make_transport

LOADER = "connex.rl.sglang_ext.connex_load"
CONTROL = "__connex_weight_sync__"

_sub = None
last_stats: dict = {}


def control_payload(registry_url, version=None, member=None, transport="engine", chunk_bytes=DEFAULT_CHUNK):
    rec = {"registry_url": registry_url, "version": version, "member": member, "transport": transport,
           "chunk_bytes": chunk_bytes}
    return [(CONTROL, torch.frombuffer(bytearray(json.dumps(rec).encode()), dtype=torch.uint8))]


def parse_control(named_tensors):
    for name, t in named_tensors:
        if name == CONTROL:
            return json.loads(bytes(t.cpu().tolist()).decode())
    return None


def _subscriber(ctl, device):
    global _sub
    if _sub is None:
        rank = int(os.environ.get("CONNEX_TP_RANK",
                                  torch.cuda.current_device() if torch.cuda.is_available() else 0))
        member = f"{ctl.get('member') or f'{socket.gethostname()}-{os.getpid()}'}/r{rank}"
        kind = ctl.get("transport") or "engine"
        kw = {"name": member} if kind in ("local", "nvlink") else {"lid": ("connex-rl", 1, rank, os.getpid())}
        _sub = WeightSubscriber(RegistryClient(ctl["registry_url"]), make_transport(kind, **kw), member,
                                device=device, chunk_bytes=ctl.get("chunk_bytes", DEFAULT_CHUNK),
                                arena="host" if kind == "engine" else "device")
    return _sub


def connex_load(model, named_tensors):
    """Custom loader: the control record names the version; the bytes come
    through the weight-sync transport.  Plain tensors load as usual."""
    global last_stats
    named_tensors = list(named_tensors)
    ctl = parse_control(named_tensors)
    if ctl is None:
        model.load_weights(named_tensors)
        return
    if os.environ.get("CONNEX_RL_DEVICE"):
        dev = torch.device(os.environ["CONNEX_RL_DEVICE"])
    elif torch.cuda.is_available():
        dev = torch.device("cuda", torch.cuda.current_device())
    else:
        dev = torch.device("cpu")
    sub = _subscriber(ctl, dev)
    m = sub.pull(ctl.get("version"))
    model.load_weights(list(sub.tensors()))
    if dev.type == "cuda":
        torch.cuda.current_stream(dev).synchronize()
    sub.commit(m.version)
    last_stats = dict(sub.stats)
