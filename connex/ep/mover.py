"""Expert weights of one EP rank, addressable by peers (reference
``connex/ep/mover.py``).

:class:`ExpertStore` holds ``layers[layer][param] -> tensor[slots, ...]``.
``describe()`` is the address book a peer needs: per layer and param the
base address and bytes per slot, plus (GPU tensors) CUDA IPC handles of the
parameter tensors.  ``apply_moves`` executes the moves whose destination
slot is on this rank:

* no live source -> ``loader(layer, expert)`` (the checkpoint; here the
  seeded random init is regenerated),
* source slot on this rank -> device copy,
* source on a peer in the same NVLink box -> the peer's tensors are mapped
  once through CUDA IPC and all rows read from that peer move in ONE launch
  of the ``copy_segments`` kernel (SM loads over NVLink) on a low-priority
  stream with a bounded CTA count, so decode kernels keep the SMs they need
  while the copy runs,
* otherwise -> one-sided reads through the transport (host memory).
"""
from __future__ import annotations

import os
import socket
import time
from collections import defaultdict
from typing import Callable, Optional

import torch


def host_id() -> str:
    try:
        boot = open("/proc/sys/kernel/random/boot_id").read().strip()
    except OSError:
        boot = ""
    return f"{socket.gethostname()}/{boot}"


class TransferError(RuntimeError):
    pass


class ExpertStore:
    def __init__(self, rank: int, layers: list, transport=None, ipc: Optional[bool] = None, copy_ctas: int = 16):
        self.rank = rank
        self.layers = [list(ps) for ps in layers]
        self.t = transport
        if self.t is not None:
            for ps in self.layers:
                for p in ps:
                    self.t.register(p)
        self.stats: dict = defaultdict(float)
        if ipc is None:
            ipc = os.environ.get("CONNEX_EP_IPC", "1") != "0"
        self.ipc = bool(ipc) and bool(self.layers) and self.layers[0][0].is_cuda
        self.copy_ctas = copy_ctas
        self._peer_map: dict = {}
        self._mapper = None
        self._stream = None

    @property
    def slots(self) -> int:
        return self.layers[0][0].shape[0] if self.layers else 0

    def row_bytes(self, layer: int, param: int) -> int:
        p = self.layers[layer][param]
        return p[0].numel() * p.element_size()

    def describe(self) -> dict:
        d = {"rank": self.rank, "url": getattr(self.t, "url", None),
             "layers": [[[p.data_ptr(), self.row_bytes(l, i)] for i, p in enumerate(ps)]
                        for l, ps in enumerate(self.layers)]}
        if self.ipc:
            from connex_b200.parallel.peer import export_tensor
            d["host"] = host_id()
            d["ipc"] = [[export_tensor(p).to_dict() for p in ps] for ps in self.layers]
        return d

    def _peer_bases(self, peer: dict) -> Optional[list]:
        """Local addresses of a same-host peer's parameter tensors (IPC), or None."""
        if not (self.ipc and peer.get("ipc") and peer.get("host") == host_id()):
            return None
        key = (peer["rank"], peer.get("url"))
        if key not in self._peer_map:
            try:
                from connex_b200.parallel.peer import PeerHandle, PeerMapper
                if self._mapper is None:
                    self._mapper = PeerMapper(self.layers[0][0].device.index)
                same = int(peer["ipc"][0][0].get("owner_pid", -1)) == os.getpid()
                self._peer_map[key] = [[(h["owner_pid"] == os.getpid() and base) or
                                        (base if same else self._mapper.open(PeerHandle.from_dict(h)))
                                        for (base, _), h in zip(rows, hs)]
                                       for rows, hs in zip(peer["layers"], peer["ipc"])]
            except Exception:
                self._peer_map[key] = None
        return self._peer_map[key]

    def apply_moves(self, moves, peers: dict, slots_per_rank: int, loader: Optional[Callable] = None,
                    timeout_ms: Optional[int] = None):
        """-> [(move, ok, error)] for the moves whose destination is on this rank."""
        t0 = time.perf_counter()
        mine = [m for m in moves if m.dst // slots_per_rank == self.rank]
        out = []
        remote = defaultdict(list)
        for m in mine:
            di = m.dst % slots_per_rank
            if m.src is None:
                if loader is None:
                    out.append((m, False, "no live source and no loader"))
                    continue
                for i, w in enumerate(loader(m.layer, m.expert)):
                    dst = self.layers[m.layer][i]
                    dst[di].copy_(w.to(dst.device, dst.dtype))
                self.stats["checkpoint_loads"] += 1
                out.append((m, True, None))
                continue
            sr, si = divmod(m.src, slots_per_rank)
            if sr == self.rank:
                for p in self.layers[m.layer]:
                    p[di].copy_(p[si])
                self.stats["local_copies"] += 1
                out.append((m, True, None))
            else:
                remote[sr].append(m)
        for sr, ms in remote.items():
            peer = peers.get(sr) if sr in peers else peers.get(str(sr))
            err = None
            if peer is None:
                err = f"no address for rank {sr}"
            else:
                try:
                    self._read_from(peer, ms, slots_per_rank, timeout_ms)
                except Exception as ex:
                    err = repr(ex)
            out.extend((m, err is None, err) for m in ms)
        dev = self.layers[0][0].device if self.layers else None
        if mine and dev is not None and dev.type == "cuda":
            torch.cuda.current_stream(dev).synchronize()
            if self._stream is not None:
                self._stream.synchronize()
        self.stats["seconds"] += time.perf_counter() - t0
        self.stats["moves"] += len(mine)
        return out

    def _read_from(self, peer: dict, moves, S: int, timeout_ms) -> None:
        bases = self._peer_bases(peer)
        if bases is not None:
            return self._copy_nvlink(bases, moves, S)
        if self.t is None:
            raise TransferError(f"no transport to reach rank {peer['rank']}")
        # one batch per destination tensor: (remote addr, byte offset in the tensor, bytes)
        per_tensor = defaultdict(list)
        for m in moves:
            si, di = m.src % S, m.dst % S
            for i, (base, rb) in enumerate(peer["layers"][m.layer]):
                per_tensor[(m.layer, i)].append((base + si * rb, di * rb, rb))
        batches = [(self.layers[l][i], ops) for (l, i), ops in per_tensor.items()]
        if hasattr(self.t, "read_many"):
            self.t.read_many(peer["url"], batches, timeout_ms=timeout_ms)
        else:
            for dst, ops in batches:
                self.t.read_batch(peer["url"], ops, dst, timeout_ms=timeout_ms)
        self.stats["bytes"] += sum(n for _, ops in batches for _, _, n in ops)

    def _copy_nvlink(self, bases, moves, S: int) -> None:
        """All rows from one peer in one copy_segments launch (bounded CTAs)."""
        from connex_b200 import ops as cxops
        dev = self.layers[0][0].device
        if self._stream is None:
            self._stream = torch.cuda.Stream(device=dev, priority=0)
        segs = []
        for m in moves:
            si, di = m.src % S, m.dst % S
            for i, p in enumerate(self.layers[m.layer]):
                rb = self.row_bytes(m.layer, i)
                segs.append((bases[m.layer][i] + si * rb, p.data_ptr() + di * rb, rb))
        total = sum(s[2] for s in segs)
        st = cxops.new_status(dev)
        self._stream.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(self._stream):
            t = torch.tensor(segs, dtype=torch.int64).to(dev, non_blocking=True)
            cxops.copy_segments(t, total, max_ctas=self.copy_ctas, status=st)
        self._stream.synchronize()
        if int(st.item()) != 0:
            raise TransferError(f"NVLink copy status {int(st.item())}")
        self.stats["bytes"] += total
        self.stats["nvlink_copies"] += len(moves)

    def checksum(self, layer: int, slot_local: int) -> float:
        """float64 sum of one slot over its params (verification helper)."""
        return float(sum(p[slot_local].double().sum().item() for p in self.layers[layer]))

    def poison(self, layer: int, slot_local: int) -> None:
        """NaN-fill a slot (negative control: a routed token would turn NaN)."""
        for p in self.layers[layer]:
            p[slot_local].fill_(float("nan"))


def moves_by_rank(moves, slots_per_rank: int) -> dict:
    """``{destination rank: [moves]}`` (reference ``connex/ep/mover.py:236``)."""
    out = defaultdict(list)
    for m in moves:
        out[m.dst // slots_per_rank].append(m)
    return dict(out)
