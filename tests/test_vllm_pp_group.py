"""vLLM PP group wrapper on CPU: two gloo ranks, the wrapped coordinator
carries the metadata and the pair links carry the tensors; tensor dicts
arrive intact and in order through the blocking and the non-blocking forms,
non-tensor values ride along, attributes the wrapper does not define reach
the wrapped coordinator, and ``install`` swaps vLLM's ``_PP`` only when
there is pipeline parallelism."""
import os
import pickle
import sys
import types

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tests.helpers import free_port


class _Coordinator:
    """The parts of vLLM's GroupCoordinator the wrapper uses (gloo world)."""

    def __init__(self, rank, world):
        self.rank_in_group, self.world_size = rank, world
        self.ranks = list(range(world))

    def send_object(self, obj, dst):
        b = torch.frombuffer(bytearray(pickle.dumps(obj)), dtype=torch.uint8)
        dist.send(torch.tensor([b.numel()]), dst)
        dist.send(b, dst)

    def recv_object(self, src):
        n = torch.zeros(1, dtype=torch.int64)
        dist.recv(n, src)
        b = torch.empty(int(n), dtype=torch.uint8)
        dist.recv(b, src)
        return pickle.loads(b.numpy().tobytes())

    def broadcast_tensor_dict(self, td=None, src=0):
        return {"delegated": True}


def _worker(rank, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=2)
        from connex.adapters.vllm.pp.group import ConnexPPGroup
        store = dist.TCPStore("127.0.0.1", port + 1, 2, rank == 0)
        grp = ConnexPPGroup(_Coordinator(rank, 2), tp_rank=0, store=store, device="cpu", kind="nccl")
        assert grp.broadcast_tensor_dict()["delegated"] and grp.ranks == [0, 1]
        g = torch.Generator().manual_seed(0)
        steps = [{"hidden_states": torch.randn(5, 16, generator=g), "residual": torch.randn(5, 16, generator=g),
                  "step": i, "note": "x" * i} for i in range(3)]
        if rank == 0:
            grp.send_tensor_dict(steps[0])
            grp.isend_tensor_dict(steps[1])
            grp.isend_tensor_dict(steps[2], dst=1)
            q.put(("sent", dict(grp.stats)))
        else:
            got = [grp.recv_tensor_dict()]
            td, handles, post = grp.irecv_tensor_dict()
            for fn in post:
                fn()
            got.append(td)
            got.append(grp.recv_tensor_dict(src=0))
            for a, b in zip(got, steps):
                assert a["step"] == b["step"] and a["note"] == b["note"]
                assert torch.equal(a["hidden_states"], b["hidden_states"])
                assert torch.equal(a["residual"], b["residual"])
            q.put(("received", dict(grp.stats)))
        dist.barrier()
        grp.links.close()
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        q.put(("error", repr(e)))
        raise


def test_tensor_dicts_cross_two_ranks_over_pair_links():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    ps = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=120) for _ in range(2)]
    for p in ps:
        p.join(60)
    assert all(p.exitcode == 0 for p in ps), res
    by = dict(res)
    assert by["sent"]["sent"] == 3 and by["sent"]["sent_tensors"] == 6
    assert by["received"]["received"] == 3


def test_install_wraps_only_pipeline_groups(monkeypatch):
    from connex.adapters.vllm.pp import group as G
    ps_mod = types.SimpleNamespace(_PP=types.SimpleNamespace(world_size=1, rank_in_group=0), _TP=None)
    pkg = types.ModuleType("vllm.distributed")
    pkg.parallel_state = ps_mod
    monkeypatch.setitem(sys.modules, "vllm", types.ModuleType("vllm"))
    monkeypatch.setitem(sys.modules, "vllm.distributed", pkg)
    assert G.install() is None and not isinstance(ps_mod._PP, G.ConnexPPGroup)

    class FakeLinks:
        device = torch.device("cpu")

    monkeypatch.setattr(G.ConnexPPGroup, "_make_links", lambda self, store, device, kind: FakeLinks())
    ps_mod._PP = types.SimpleNamespace(world_size=2, rank_in_group=1)
    ps_mod._TP = types.SimpleNamespace(rank_in_group=3)
    grp = G.install()
    assert isinstance(ps_mod._PP, G.ConnexPPGroup) and grp.me == "cxvpp1.tp3" and grp.name(0) == "cxvpp0.tp3"
    assert G.install() is grp                       # idempotent


def test_plugin_wraps_the_group_after_model_parallel_init(monkeypatch):
    from connex.adapters.vllm import plugin
    from connex.adapters.vllm.pp import group as G
    calls = []
    ps_mod = types.SimpleNamespace(_PP=None, _TP=None)

    def initialize_model_parallel(tp=1, pp=1):
        calls.append((tp, pp))
        ps_mod._PP = types.SimpleNamespace(world_size=pp, rank_in_group=0)
    ps_mod.initialize_model_parallel = initialize_model_parallel
    pkg = types.ModuleType("vllm.distributed")
    pkg.parallel_state = ps_mod
    monkeypatch.setitem(sys.modules, "vllm", types.ModuleType("vllm"))
    monkeypatch.setitem(sys.modules, "vllm.distributed", pkg)

    class FakeLinks:
        device = torch.device("cpu")
    monkeypatch.setattr(G.ConnexPPGroup, "_make_links", lambda self, store, device, kind: FakeLinks())
    monkeypatch.setenv("CONNEX_PP_GROUP", "1")
    plugin.register()
    plugin.register()                                 # once only
    ps_mod.initialize_model_parallel(1, 2)
    assert calls == [(1, 2)] and isinstance(ps_mod._PP, G.ConnexPPGroup)
