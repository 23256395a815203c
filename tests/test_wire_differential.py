"""Differential wire test: this package's PP wire codec against the
reference's own (``connex/pp/wire.py`` of the reference as installed under
``baseline/_ref``, loaded by path: it is pure stdlib), driven by the same
generated inputs.  Every byte either side puts on the wire must be equal,
and each side must decode the other's frames to the same values: layouts
(every dtype code, 0-4 dims, unicode keys), G2 tails, data signals (with
and without the correlation field), acks and correlation ids.  Without the
installed reference the committed golden frames (produced by the
reference's codec) are checked instead."""
import importlib.util
import json
import struct
import sys
from pathlib import Path

import pytest
from hypothesis import given, settings
from hypothesis import strategies as st

from connex.pp import wire

ROOT = Path(__file__).resolve().parents[1]
REF_WIRE = ROOT / "baseline" / "_ref" / "connex" / "pp" / "wire.py"
GOLDEN = Path(__file__).resolve().parent / "data" / "wire_golden.json"


def _load_ref():
    if not REF_WIRE.exists():
        return None
    spec = importlib.util.spec_from_file_location("reference_pp_wire", REF_WIRE)
    mod = importlib.util.module_from_spec(spec)
    sys.modules["reference_pp_wire"] = mod            # its dataclasses look their module up
    spec.loader.exec_module(mod)
    return mod


REF = _load_ref()
need_ref = pytest.mark.skipif(REF is None, reason="the reference is not installed under baseline/_ref")

keys = st.text(min_size=0, max_size=24)
dtypes = st.sampled_from(wire.DT_NAMES)
shapes = st.lists(st.integers(0, 1 << 40), min_size=0, max_size=4).map(tuple)
u64 = st.integers(0, (1 << 64) - 1)
entries = st.lists(st.tuples(keys, dtypes, shapes, u64, u64), min_size=0, max_size=12)
blobs = st.binary(max_size=300)


@need_ref
@settings(max_examples=300, deadline=None)
@given(entries)
def test_layout_bytes_and_cross_decode(layout):
    mine, theirs = wire.encode_layout(layout), REF.encode_layout(layout)
    assert mine == theirs
    assert [tuple(x) for x in wire.decode_layout(theirs)] == [tuple(x) for x in REF.decode_layout(mine)] == \
        [tuple(x) for x in layout]


@need_ref
def test_unknown_dtype_has_no_layout_on_either_side():
    bad = [("x", "complex64", (1,), 0, 8)]
    assert wire.encode_layout(bad) is None and REF.encode_layout(bad) is None


@need_ref
@settings(max_examples=300, deadline=None)
@given(u64, blobs, blobs, blobs, blobs)
def test_g2_tail(token, layout_b, ack_ep, origin, nt):
    ack_ep = ack_ep.decode("latin-1").encode()[:200]
    ack_ep = bytes(b & 0x7F for b in ack_ep)              # endpoint addresses are ASCII
    origin = bytes(b & 0x7F for b in origin)
    mine = wire.encode_g2(token, layout_b, ack_ep, origin, nt)
    assert mine == REF.encode_g2(token, layout_b, ack_ep, origin, nt)
    assert tuple(wire.decode_g2(mine[2:])) == tuple(REF.decode_g2(mine[2:]))


@need_ref
@settings(max_examples=300, deadline=None)
@given(u64, u64, st.text(max_size=60), u64, blobs)
def test_signal(src, total, url, corr, tail):
    ub = url.encode()
    mine = wire.encode_signal(src, total, ub, corr, tail)
    assert mine == REF.encode_signal(src, total, ub, corr, tail)
    a, b = wire.decode_signal(mine), REF.decode_signal(mine)
    assert (a.src_ptr, a.total, a.url, a.corr, a.tail) == (b.src_ptr, b.total, b.url, b.corr, b.tail)
    assert wire.signal_corr(mine) == REF.signal_corr(mine) == corr
    old = wire.WIRE_MAGIC + struct.pack("!QQI", src, total, len(ub)) + ub     # before the corr field
    assert wire.decode_signal(old).corr is None and REF.decode_signal(old).corr is None


@need_ref
@settings(max_examples=200, deadline=None)
@given(u64, st.integers(0, (1 << 32) - 1), st.integers(0, (1 << 32) - 1), blobs)
def test_ack_and_corr(token, inc, seq, junk):
    assert wire.encode_ack(token) == REF.encode_ack(token)
    assert wire.decode_ack(wire.encode_ack(token)) == REF.decode_ack(wire.encode_ack(token)) == token
    assert wire.decode_ack(junk) == REF.decode_ack(junk)
    c = wire.make_corr(inc, seq)
    assert wire.corr_incarnation(c) == REF.corr_incarnation(c) and wire.corr_seq(c) == REF.corr_seq(c)


@need_ref
@settings(max_examples=100, deadline=None)
@given(st.lists(st.tuples(keys, dtypes, shapes.filter(lambda s: len(s) <= 3)), min_size=1, max_size=8),
       st.lists(st.integers(0, 1 << 30), min_size=8, max_size=8))
def test_codec_places_tensors_like_the_reference(specs, sizes):
    specs = tuple(specs)
    sizes = sizes[:len(specs)]
    m, r = wire.LayoutCodec().layout_for(specs, sizes), REF.LayoutCodec().layout_for(specs, sizes)
    assert [tuple(x) for x in m[0]] == [tuple(x) for x in r[0]] and m[1] == r[1] and m[2] == r[2]


def test_golden_frames():
    """Frames the reference's codec produced (committed): this codec writes
    the same bytes and reads them back."""
    g = json.loads(GOLDEN.read_text())
    for case in g["layouts"]:
        layout = [(k, dt, tuple(sh), off, nb) for k, dt, sh, off, nb in case["layout"]]
        assert wire.encode_layout(layout).hex() == case["bytes"]
        assert [tuple(x) for x in wire.decode_layout(bytes.fromhex(case["bytes"]))] == layout
    for case in g["signals"]:
        b = wire.encode_signal(case["src"], case["total"], case["url"].encode(), case["corr"],
                               bytes.fromhex(case["tail"]))
        assert b.hex() == case["bytes"]
        s = wire.decode_signal(b)
        assert (s.src_ptr, s.total, s.url, s.corr) == (case["src"], case["total"], case["url"], case["corr"])
    for case in g["g2"]:
        b = wire.encode_g2(case["token"], bytes.fromhex(case["layout"]), case["ack_ep"].encode(),
                           case["origin"].encode(), bytes.fromhex(case["nt"]))
        assert b.hex() == case["bytes"]
    for case in g["acks"]:
        assert wire.encode_ack(case["token"]).hex() == case["bytes"]
