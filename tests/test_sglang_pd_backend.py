"""SGLang ``connex`` transfer backend without SGLang: the engine surface the
Mooncake KV manager calls (session ids, batched writes through the native
engine, failures, probes), plugin registration against stand-in SGLang
modules (closed enum extended, ``get_kv_class`` routed), and on a GPU the
NVLink path (IPC region record + one copy kernel per batch)."""
import enum
import sys
import types

import pytest
import torch

from connex.adapters.sglang import pd_backend
from connex.adapters.sglang.pd_backend import INVALID, ConnexTransferEngine, extend_enum


class FakeHandle:
    def __init__(self, ok):
        self.ok = ok

    def wait(self, timeout_ms=None):
        if not self.ok:
            raise RuntimeError("peer failed")
        return True


class FakeEngine:
    def __init__(self, model, stage, shard, replica, **kw):
        self.local_url = f"{kw['listen_ip']}:{kw['port']}#{model}|{stage}|{shard}|{replica}"
        self.connected, self.puts, self.regions, self.fail_after = [], [], {}, None

    def register_memory(self, ptr, n):
        self.regions[ptr] = n
        return 0

    def unregister_memory(self, ptr):
        self.regions.pop(ptr, None)
        return 0

    def put_async(self, url, src, dst, n, timeout_ms=None):
        self.puts.append((url, src, dst, n))
        return FakeHandle(self.fail_after is None or len(self.puts) <= self.fail_after)

    def connect(self, url):
        self.connected.append(url)
        if "dead" in url:
            raise RuntimeError("unreachable")


def _engine(monkeypatch, role="prefill", port=5000, shm=None):
    monkeypatch.setenv("CONNEX_RS_PORT", str(port))
    kw = {"shm_dir": str(shm)} if shm else {}
    return ConnexTransferEngine("10.0.0.1", role, gpu_id=0, engine_cls=FakeEngine, **kw)


def test_session_id_and_peer_identity(monkeypatch):
    e = _engine(monkeypatch)
    assert e.url == "10.0.0.1:5000#sglang-pd|1000|0|5000" and e.get_session_id() == "10.0.0.1:5000"
    assert e.peer_url("10.0.0.2:5123") == "10.0.0.2:5123#sglang-pd|1001|0|5123"
    assert e.peer_url("h:1#m|1|0|1") == "h:1#m|1|0|1"
    assert e.batch_register([1, 2], [10, 20]) == 0 and e.engine.regions == {1: 10, 2: 20}
    assert e.batch_deregister([1]) == 0 and e.engine.regions == {2: 20}


def test_host_writes_posted_together_and_failures_reported(monkeypatch):
    e = _engine(monkeypatch)
    n = 1 << 16
    assert e.batch_transfer_sync("10.0.0.2:5123", [1, 2, 3], [11, 12, 13], [n] * 3) == 0
    assert [p[1:] for p in e.engine.puts] == [(1, 11, n), (2, 12, n), (3, 13, n)]
    assert e.transfer_sync("10.0.0.2:5123", 4, 14, 100) == 0
    e.engine.puts, e.engine.fail_after = [], 1
    assert e.batch_transfer_sync("10.0.0.2:5123", [1, 2], [11, 12], [n, n]) == pd_backend.PEER_FAILED
    assert e.send_probe("10.0.0.2:1") == 0 and e.send_probe("dead:1") == -1
    assert e.engine.connected[0] == "10.0.0.2:1#sglang-pd|1001|0|1"
    # GPU pages with no NVLink route to the peer are refused, not sent through host RMA
    e.device_regions.append((1, 1 << 20))
    assert e.batch_transfer_sync("10.0.0.2:5123", [1], [2], [100]) == INVALID


def test_extend_enum_plain_and_str_enums():
    class TB(enum.Enum):
        MOONCAKE = "mooncake"

    class SB(str, enum.Enum):
        A = "a"

    m = extend_enum(TB, "CONNEX", "connex")
    assert TB("connex") is m is TB.CONNEX and m.name == "CONNEX" and list(TB)[-1] is m
    assert extend_enum(TB, "CONNEX", "connex") is m
    s = extend_enum(SB, "B", "b")
    assert SB("b") is s and s == "b" and isinstance(s, str)


def _fake_sglang(monkeypatch):
    """The SGLang names the plugin touches, as stand-in modules."""
    class TransferBackend(enum.Enum):
        MOONCAKE = "mooncake"

    class KVClassType(enum.Enum):
        KVARGS, MANAGER, SENDER, RECEIVER, BOOTSTRAP_SERVER = range(5)

    class DisaggregationMode(enum.Enum):
        PREFILL, DECODE = "prefill", "decode"

    class MooncakeKVManager:
        def __init__(self, mode, gpu_id):
            self.disaggregation_mode, self.local_ip = mode, "127.0.0.1"
            self.kv_args = types.SimpleNamespace(gpu_id=gpu_id, engine_rank=0)
            self.init_engine()

        def init_engine(self):
            self.engine = "mooncake"

    conn = types.ModuleType("sglang.srt.disaggregation.mooncake.conn")
    conn.MooncakeKVManager = MooncakeKVManager
    for n in ("MooncakeKVSender", "MooncakeKVReceiver", "MooncakeKVBootstrapServer"):
        setattr(conn, n, type(n, (), {}))
    du = types.ModuleType("sglang.srt.disaggregation.utils")
    du.TransferBackend, du.KVClassType, du.DisaggregationMode = TransferBackend, KVClassType, DisaggregationMode
    du.get_kv_class = lambda backend, kind: {KVClassType.MANAGER: MooncakeKVManager}.get(kind)
    base = types.ModuleType("sglang.srt.disaggregation.base")
    base.KVArgs = type("KVArgs", (), {})
    choices = types.ModuleType("sglang.srt.arg_groups.choices")
    choices.DISAGG_TRANSFER_BACKEND_CHOICES = ["mooncake"]
    choices.add_disagg_transfer_backend_choices = choices.DISAGG_TRANSFER_BACKEND_CHOICES.extend
    user = types.ModuleType("fake_sglang_user")          # imported get_kv_class by name earlier
    user.get_kv_class = du.get_kv_class
    mods = {"sglang": types.ModuleType("sglang"), "sglang.srt": types.ModuleType("sglang.srt"),
            "sglang.srt.disaggregation": types.ModuleType("sglang.srt.disaggregation"),
            "sglang.srt.disaggregation.mooncake": types.ModuleType("sglang.srt.disaggregation.mooncake"),
            "sglang.srt.disaggregation.mooncake.conn": conn, "sglang.srt.disaggregation.utils": du,
            "sglang.srt.disaggregation.base": base, "sglang.srt.arg_groups": types.ModuleType("sglang.srt.arg_groups"),
            "sglang.srt.arg_groups.choices": choices, "fake_sglang_user": user}
    for k, v in mods.items():
        monkeypatch.setitem(sys.modules, k, v)
    return du, conn, choices, user


def test_plugin_registers_the_backend(monkeypatch):
    du, conn, choices, user = _fake_sglang(monkeypatch)
    made = []
    monkeypatch.setattr(pd_backend, "get_engine", lambda host, role, gpu: made.append((host, role, gpu)) or "cx")
    pd_backend.register()
    pd_backend.register()                                   # idempotent
    tb = du.TransferBackend("connex")
    assert tb is du.TransferBackend.CONNEX and choices.DISAGG_TRANSFER_BACKEND_CHOICES == ["mooncake", "connex"]
    mgr = du.get_kv_class(tb, du.KVClassType.MANAGER)
    assert issubclass(mgr, conn.MooncakeKVManager) and mgr is not conn.MooncakeKVManager
    assert du.get_kv_class(tb, du.KVClassType.KVARGS).__name__ == "KVArgs"
    assert du.get_kv_class(du.TransferBackend.MOONCAKE, du.KVClassType.MANAGER) is conn.MooncakeKVManager
    assert user.get_kv_class is du.get_kv_class
    m = mgr(du.DisaggregationMode.DECODE, 3)
    assert m.engine == "cx" and made == [("127.0.0.1", "decode", 3)]


@pytest.mark.gpu
def test_nvlink_batch_is_one_copy_into_the_peer_regions(monkeypatch, tmp_path):
    dec = _engine(monkeypatch, "decode", 6000, tmp_path)
    pre = _engine(monkeypatch, "prefill", 6100, tmp_path)
    dst = torch.zeros(64, 4096, dtype=torch.bfloat16, device="cuda")
    src = torch.randn(64, 4096, device="cuda").bfloat16()
    dec.register(dst.data_ptr(), dst.numel() * 2)
    pre.register(src.data_ptr(), src.numel() * 2)
    assert (tmp_path / "connex-sglpd-10.0.0.1_6000.json").exists()
    page = 4096 * 2
    order = [5, 0, 63, 17]                    # scattered pages, like KV page indices
    srcs = [src.data_ptr() + i * page for i in range(4)]
    dsts = [dst.data_ptr() + j * page for j in order]
    assert pre.batch_transfer_sync(dec.session_id, srcs, dsts, [page] * 4) == 0
    torch.cuda.synchronize()
    for i, j in enumerate(order):
        assert torch.equal(dst[j], src[i])
    assert pre.stats["nvlink_batches"] == 1 and pre.engine.puts == []
    # an address outside the peer's registered regions is refused
    assert pre.batch_transfer_sync(dec.session_id, srcs[:1], [dst.data_ptr() + dst.numel() * 2], [page]) == INVALID
    dec.close()
    pre.close()
