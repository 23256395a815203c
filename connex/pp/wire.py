"""PP data-plane wire format (pure stdlib, byte-compatible with the reference).

Data signal (one ZeroMQ frame, DEALER -> ROUTER)::

    b"CONNEXTE" | !Q src_ptr | !Q total | !I url_len | url | !Q corr | tail

``total`` bytes at ``src_ptr`` in the sender's registered memory at
transfer-engine segment ``url`` are pulled by the receiver with one
one-sided read.  ``tail`` is empty (host payload), ``b"G1" + pickle`` (legacy
header) or ``b"G2" + !QIIHH(token, layout_len, nt_len, ack_ep_len,
origin_len) + layout + ack_ep + origin + nt``.  The G2 ``layout`` is
``!H n`` then, per tensor, ``!HBB(keylen, dtype code, ndim) key
!{ndim}q(shape) !QQ(offset, nbytes)``; tensors sit at 256-byte aligned
offsets.  The ack is ``b"CXACK" + !Q token``.  ``corr = incarnation << 32 |
seq``.  (Reference: ``connex/pp/wire.py:8-207``.)

The dtype code table is append-only: codes travel on the wire.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass
from typing import List, Optional, Tuple

WIRE_MAGIC = b"CONNEXTE"
ACK_MARK = b"CXACK"
ACK = struct.Struct("!Q")
SIG_FIXED = struct.Struct("!QQI")
CORR = struct.Struct("!Q")
HOST_HDR = struct.Struct("!Qd")
G2 = struct.Struct("!QIIHH")
TAG_G1 = b"G1"
TAG_G2 = b"G2"
WIRE_VERSION = 2

KEY_ORIGIN = "__stage0_endpoint__"
KEY_SEND_TS = "__send_timestamp__"

DT_NAMES = ("float32", "float16", "bfloat16", "float64", "int64", "int32",
            "int16", "int8", "uint8", "bool", "float8_e4m3fn", "float8_e5m2")
DT_CODE = {name: code for code, name in enumerate(DT_NAMES)}

_LAYOUT_N = struct.Struct("!H")
_LAYOUT_ENTRY = struct.Struct("!HBB")
_LAYOUT_SPAN = struct.Struct("!QQ")


def align(n: int, a: int = 256) -> int:
    return -(-n // a) * a


LayoutEntry = Tuple[str, str, tuple, int, int]  # key, dtype name, shape, offset, nbytes


def encode_layout(layout: List[LayoutEntry]) -> Optional[bytes]:
    """Encode a G2 layout; ``None`` if some dtype has no wire code."""
    out = bytearray(_LAYOUT_N.pack(len(layout)))
    for key, dt, shape, off, nb in layout:
        code = DT_CODE.get(dt)
        if code is None:
            return None
        kb = key.encode()
        out += _LAYOUT_ENTRY.pack(len(kb), code, len(shape))
        out += kb
        out += struct.pack(f"!{len(shape)}q", *shape)
        out += _LAYOUT_SPAN.pack(off, nb)
    return bytes(out)


def decode_layout(b: bytes) -> List[LayoutEntry]:
    (n,) = _LAYOUT_N.unpack_from(b, 0)
    pos = _LAYOUT_N.size
    out = []
    for _ in range(n):
        klen, code, ndim = _LAYOUT_ENTRY.unpack_from(b, pos)
        pos += _LAYOUT_ENTRY.size
        key = b[pos:pos + klen].decode()
        pos += klen
        shape = struct.unpack_from(f"!{ndim}q", b, pos)
        pos += 8 * ndim
        off, nb = _LAYOUT_SPAN.unpack_from(b, pos)
        pos += _LAYOUT_SPAN.size
        out.append((key, DT_NAMES[code], tuple(shape), off, nb))
    return out


def encode_g2(token: int, layout_b: bytes, ack_ep: bytes, origin: bytes, nt_b: bytes) -> bytes:
    return b"".join((TAG_G2, G2.pack(token, len(layout_b), len(nt_b), len(ack_ep), len(origin)),
                     layout_b, ack_ep, origin, nt_b))


def decode_g2(body: bytes):
    """``body`` follows the ``G2`` tag -> (token, layout bytes, ack_ep, origin, nt bytes)."""
    token, ll, nl, al, ol = G2.unpack_from(body, 0)
    p = G2.size
    layout_b = body[p:p + ll]
    p += ll
    ack_ep = body[p:p + al].decode()
    p += al
    origin = body[p:p + ol].decode()
    p += ol
    return token, layout_b, ack_ep, origin, body[p:p + nl]


class LayoutCodec:
    """Bounded caches: (keys, dtypes, shapes) -> layout on the sender, layout
    bytes -> parsed layout on the receiver (no re-encoding in steady state)."""

    def __init__(self, cap: int = 512):
        self.cap = cap
        self.enc: dict = {}
        self.dec: dict = {}

    def layout_for(self, key, sizes):
        hit = self.enc.get(key)
        if hit is None:
            layout, total = [], 0
            for (name, dt, shape), nb in zip(key, sizes):
                layout.append((name, dt, shape, total, nb))
                total = align(total + nb)
            hit = (layout, total, encode_layout(layout))
            if len(self.enc) >= self.cap:
                self.enc.clear()
            self.enc[key] = hit
        return hit

    def parse(self, b: bytes):
        hit = self.dec.get(b)
        if hit is None:
            hit = decode_layout(b)
            if len(self.dec) >= self.cap:
                self.dec.clear()
            self.dec[b] = hit
        return hit


def encode_signal(src_ptr: int, total: int, url: bytes, corr: int, tail: bytes = b"") -> bytes:
    return b"".join((WIRE_MAGIC, SIG_FIXED.pack(src_ptr, total, len(url)), url, CORR.pack(corr), tail))


@dataclass
class Signal:
    src_ptr: int
    total: int
    url: str
    corr: Optional[int]
    tail: bytes

    @property
    def tag(self) -> bytes:
        return self.tail[:2]


def decode_signal(data: bytes) -> Signal:
    if not data.startswith(WIRE_MAGIC):
        raise ValueError("not a CONNEXTE signal")
    meta = data[len(WIRE_MAGIC):]
    if len(meta) < SIG_FIXED.size:
        raise ValueError("Invalid metadata length")
    src, total, ul = SIG_FIXED.unpack_from(meta, 0)
    if len(meta) < SIG_FIXED.size + ul:
        raise ValueError("Incomplete sender URL")
    url = meta[SIG_FIXED.size:SIG_FIXED.size + ul].decode()
    rest = meta[SIG_FIXED.size + ul:]
    if len(rest) >= CORR.size:
        return Signal(src, total, url, CORR.unpack_from(rest, 0)[0], rest[CORR.size:])
    return Signal(src, total, url, None, b"")


def signal_corr(sig: bytes) -> int:
    ul = struct.unpack_from("!I", sig, len(WIRE_MAGIC) + 16)[0]
    return CORR.unpack_from(sig, len(WIRE_MAGIC) + SIG_FIXED.size + ul)[0]


def encode_ack(token: int) -> bytes:
    return ACK_MARK + ACK.pack(token)


def decode_ack(data: bytes) -> Optional[int]:
    if data.startswith(ACK_MARK) and len(data) >= len(ACK_MARK) + ACK.size:
        return ACK.unpack_from(data, len(ACK_MARK))[0]
    return None


def make_corr(incarnation: int, seq: int) -> int:
    return ((incarnation & 0xFFFFFFFF) << 32) | (seq & 0xFFFFFFFF)


def corr_incarnation(corr: int) -> int:
    return corr >> 32


def corr_seq(corr: int) -> int:
    return corr & 0xFFFFFFFF


# ---- host payload (tail = b"") ------------------------------------------------
def encode_host_payload(tensors: dict, non_tensors: dict, send_ts: float) -> bytes:
    """``!Qd(tensor_len, send_ts) + safetensors(tensors) + pickle(non_tensors)``."""
    import pickle
    blob = b""
    if tensors:
        from safetensors.torch import save as _st_save  # optional dependency
        blob = _st_save({k: v.contiguous().cpu() for k, v in tensors.items()})
    return HOST_HDR.pack(len(blob), send_ts) + blob + pickle.dumps(non_tensors)


def decode_host_payload(data: bytes):
    import pickle
    n, ts = HOST_HDR.unpack_from(data, 0)
    p = HOST_HDR.size
    tensors = {}
    if n:
        from safetensors.torch import load as _st_load
        tensors = _st_load(data[p:p + n])
    return tensors, pickle.loads(data[p + n:]), ts
