"""PP data-plane wire format (pure stdlib).

The bytes must match the reference's endpoints, so the layout is fixed;
the code here is organised around three record types, each with one
``pack`` and one ``unpack``:

:class:`Signal` -- one ZeroMQ frame, DEALER -> ROUTER::

    b"CONNEXTE" | !Q src_ptr | !Q total | !I url_len | url | !Q corr | tail

  ``total`` bytes at ``src_ptr`` in the sender's registered memory (at
  transfer-engine segment ``url``) are pulled by the receiver with one
  one-sided read, or travel inline / over a link.  A signal without the
  ``corr`` field decodes with ``corr=None``.  ``corr = incarnation << 32 |
  seq``.

:class:`G2` -- the ``tail`` of a signal: ``b"G2" + !QIIHH(token,
  layout_len, nt_len, ack_ep_len, origin_len) + layout + ack_ep + origin +
  nt`` (``b"G1" + pickle`` is the legacy tail; an empty tail is a host
  payload).

:class:`Layout` -- the tensors of a step inside the payload: ``!H n`` then
  per tensor ``!HBB(key_len, dtype code, ndim) key !{ndim}q(shape)
  !QQ(offset, nbytes)``; tensors start on 256-byte boundaries.

The ack of a ring slot is ``b"CXACK" + !Q token``.  The dtype code table is
append-only: codes travel on the wire.  Byte compatibility with the
reference's ``connex/pp/wire.py:8-207`` is checked by a differential test.
"""
from __future__ import annotations

import collections
import struct
from dataclasses import dataclass
from typing import List, NamedTuple, Optional, Sequence, Tuple

WIRE_MAGIC = b"CONNEXTE"
ACK_MARK = b"CXACK"
TAG_G1 = b"G1"
TAG_G2 = b"G2"
WIRE_VERSION = 2
ALIGN = 256

KEY_ORIGIN = "__stage0_endpoint__"
KEY_SEND_TS = "__send_timestamp__"

DT_NAMES = ("float32", "float16", "bfloat16", "float64", "int64", "int32",
            "int16", "int8", "uint8", "bool", "float8_e4m3fn", "float8_e5m2")
DT_CODE = {name: code for code, name in enumerate(DT_NAMES)}

_U64 = struct.Struct("!Q")
_SIG_HEAD = struct.Struct("!QQI")           # src_ptr, total, url_len
_G2_HEAD = struct.Struct("!QIIHH")          # token, layout_len, nt_len, ack_ep_len, origin_len
_N = struct.Struct("!H")
_ENTRY = struct.Struct("!HBB")              # key_len, dtype code, ndim
_SPAN = struct.Struct("!QQ")                # offset, nbytes
HOST_HDR = struct.Struct("!Qd")             # tensor blob length, send timestamp

# older names of the fixed parts, kept for callers that build frames by hand
SIG_FIXED = _SIG_HEAD
CORR = _U64
ACK = _U64
G2_FIXED = _G2_HEAD


def align(n: int, a: int = ALIGN) -> int:
    return -(-n // a) * a


# ---------------------------------------------------------------- layout
class Slot(NamedTuple):
    """One tensor of a step payload."""
    key: str
    dtype: str
    shape: tuple
    offset: int
    nbytes: int


LayoutEntry = Tuple[str, str, tuple, int, int]  # a Slot as a plain tuple


class Layout:
    """Slots of a payload; ``pack`` returns None when a dtype has no code."""

    @staticmethod
    def pack(slots: Sequence[LayoutEntry]) -> Optional[bytes]:
        parts = [_N.pack(len(slots))]
        for key, dt, shape, off, nb in slots:
            code = DT_CODE.get(dt)
            if code is None:
                return None
            kb = key.encode()
            parts += (_ENTRY.pack(len(kb), code, len(shape)), kb, struct.pack(f"!{len(shape)}q", *shape),
                      _SPAN.pack(off, nb))
        return b"".join(parts)

    @staticmethod
    def unpack(b: bytes) -> List[Slot]:
        mv = memoryview(b)
        (n,), pos = _N.unpack_from(mv, 0), _N.size
        slots = []
        for _ in range(n):
            klen, code, ndim = _ENTRY.unpack_from(mv, pos)
            pos += _ENTRY.size
            key = bytes(mv[pos:pos + klen]).decode()
            pos += klen
            shape = struct.unpack_from(f"!{ndim}q", mv, pos)
            pos += 8 * ndim
            off, nb = _SPAN.unpack_from(mv, pos)
            pos += _SPAN.size
            slots.append(Slot(key, DT_NAMES[code], tuple(shape), off, nb))
        return slots

    @staticmethod
    def place(specs, sizes) -> Tuple[List[Slot], int]:
        """Slots for tensors ``specs`` ((key, dtype, shape), ...) of ``sizes``
        bytes, each on a 256-byte boundary; returns (slots, payload bytes)."""
        slots, at = [], 0
        for (key, dt, shape), nb in zip(specs, sizes):
            slots.append(Slot(key, dt, shape, at, nb))
            at = align(at + nb)
        return slots, at


class LayoutCodec:
    """LRU caches of both directions: a step's (key, dtype, shape) tuple ->
    (slots, payload bytes, packed layout) on the sender, packed layout ->
    slots on the receiver; steady-state steps neither pack nor parse."""

    def __init__(self, cap: int = 512):
        self.cap = cap
        self.enc: "collections.OrderedDict" = collections.OrderedDict()
        self.dec: "collections.OrderedDict" = collections.OrderedDict()

    def _get(self, cache, key, make):
        hit = cache.get(key)
        if hit is None:
            hit = cache[key] = make()
            if len(cache) > self.cap:
                cache.popitem(last=False)
        else:
            cache.move_to_end(key)
        return hit

    def layout_for(self, specs, sizes):
        def make():
            slots, total = Layout.place(specs, sizes)
            return slots, total, Layout.pack(slots)
        return self._get(self.enc, specs, make)

    def parse(self, b: bytes) -> List[Slot]:
        return self._get(self.dec, b, lambda: Layout.unpack(b))


# ---------------------------------------------------------------- G2 tail
class G2(NamedTuple):
    token: int
    layout: bytes
    ack_ep: bytes
    origin: bytes
    nt: bytes

    def pack(self) -> bytes:
        return b"".join((TAG_G2, _G2_HEAD.pack(self.token, len(self.layout), len(self.nt), len(self.ack_ep),
                                               len(self.origin)), self.layout, self.ack_ep, self.origin, self.nt))

    @classmethod
    def unpack(cls, body: bytes) -> "G2":
        """``body``: the tail after the two tag bytes."""
        token, ll, nl, al, ol = _G2_HEAD.unpack_from(body, 0)
        a = _G2_HEAD.size
        b = a + ll
        c = b + al
        d = c + ol
        return cls(token, body[a:b], body[b:c], body[c:d], body[d:d + nl])


# ---------------------------------------------------------------- signal
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

    @staticmethod
    def pack(src_ptr: int, total: int, url: bytes, corr: int, tail: bytes = b"") -> bytes:
        return b"".join((WIRE_MAGIC, _SIG_HEAD.pack(src_ptr, total, len(url)), url, _U64.pack(corr), tail))

    @classmethod
    def unpack(cls, data: bytes) -> "Signal":
        if data[:len(WIRE_MAGIC)] != WIRE_MAGIC:
            raise ValueError("not a CONNEXTE signal")
        p = len(WIRE_MAGIC)
        if len(data) < p + _SIG_HEAD.size:
            raise ValueError("Invalid metadata length")
        src, total, ul = _SIG_HEAD.unpack_from(data, p)
        p += _SIG_HEAD.size
        if len(data) < p + ul:
            raise ValueError("Incomplete sender URL")
        url = data[p:p + ul].decode()
        p += ul
        if len(data) < p + _U64.size:                     # a signal from before the corr field
            return cls(src, total, url, None, b"")
        return cls(src, total, url, _U64.unpack_from(data, p)[0], data[p + _U64.size:])

    @staticmethod
    def corr_of(sig: bytes) -> int:
        """The correlation id of a packed signal, without unpacking the rest."""
        ul = struct.unpack_from("!I", sig, len(WIRE_MAGIC) + 16)[0]
        return _U64.unpack_from(sig, len(WIRE_MAGIC) + _SIG_HEAD.size + ul)[0]


# ---------------------------------------------------------------- acks, ids
def encode_ack(token: int) -> bytes:
    return ACK_MARK + _U64.pack(token)


def decode_ack(data: bytes) -> Optional[int]:
    """The token of an ack frame, None for any other frame."""
    n = len(ACK_MARK)
    if data[:n] != ACK_MARK or len(data) < n + _U64.size:
        return None
    return _U64.unpack_from(data, n)[0]


def make_corr(incarnation: int, seq: int) -> int:
    return ((incarnation & 0xFFFFFFFF) << 32) | (seq & 0xFFFFFFFF)


def corr_incarnation(corr: int) -> int:
    return corr >> 32


def corr_seq(corr: int) -> int:
    return corr & 0xFFFFFFFF


# ------------------------------------------------- function-style entry points
def encode_layout(layout: Sequence[LayoutEntry]) -> Optional[bytes]:
    return Layout.pack(layout)


def decode_layout(b: bytes) -> List[Slot]:
    return Layout.unpack(b)


def encode_g2(token: int, layout_b: bytes, ack_ep: bytes, origin: bytes, nt_b: bytes) -> bytes:
    return G2(token, layout_b, ack_ep, origin, nt_b).pack()


def decode_g2(body: bytes):
    """(token, layout, ack_ep (str), origin (str), nt) of a G2 tail body."""
    g = G2.unpack(body)
    return g.token, g.layout, g.ack_ep.decode(), g.origin.decode(), g.nt


encode_signal = Signal.pack
decode_signal = Signal.unpack
signal_corr = Signal.corr_of


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
