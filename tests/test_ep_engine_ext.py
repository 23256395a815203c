"""EP engine glue without a running engine: the ``connex_ep_*`` RPCs write a
placement view into tensors shaped like vLLM's ``EplbModelState`` and
SGLang's ``ExpertLocationMetadata`` (in place), an ``EPController`` drives two
in-process "ranks" through an HTTP ``/collective_rpc`` stand-in (describe,
apply, async moves, checksums), and the SGLang control endpoint runs commands
on a scheduler stand-in between its steps, also with two gloo TP ranks."""
import json
import queue
import threading
import time
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer

import pytest
import torch

from connex.ep import EPController, PlacementTable, logical_to_physical
from connex.ep import sglang_ext
from connex.ep.engine_ext import EngineMaps, EPWorkerCore, slot_sums

E, R, S, L, H = 4, 2, 4, 2, 3


def _naive_sums(layers, slots, S):
    return {str(p): float(sum(w[p % S].double().sum().item() for ps in layers for w in ps)) for p in slots}


def test_slot_sums_match_naive_loop_for_every_chunk_size():
    g = torch.Generator().manual_seed(0)
    layers = [[torch.randn(8, 16, 4, generator=g).half(), torch.randn(8, 5, generator=g)] for _ in range(3)]
    slots = [9, 10, 15]
    want = _naive_sums(layers, slots, 8)
    for budget in (1, 512, 1 << 30):
        got = slot_sums(layers, slots, 8, budget=budget)
        assert got.keys() == want.keys()
        for k in want:
            assert got[k] == pytest.approx(want[k], rel=1e-12, abs=1e-9)
    assert slot_sums(layers, [], 8) == {}


# --------------------------------------------------------------- vLLM layout
def _vllm_state(rows, W):
    p2l = torch.tensor(rows)
    l2p = torch.full((L, E, W), -1, dtype=torch.long)
    cnt = torch.zeros(L, E, dtype=torch.long)
    for l in range(L):
        for p, e in enumerate(rows[l]):
            if e >= 0:
                l2p[l, e, cnt[l, e]] = p
                cnt[l, e] += 1
    return p2l, l2p, cnt


class _MoELayer:
    def __init__(self, ws):
        self.ws = ws

    def get_expert_weights(self):
        return self.ws


class _Rank(EPWorkerCore):
    """A vLLM-like worker: its EplbModelState maps plus expert weights
    ``[S, H, H]`` per layer, slot ``p`` filled with ``expert + 10 * layer``."""

    def __init__(self, rank, rows, W):
        self.rank = rank
        self.p2l, self.l2p, self.cnt = _vllm_state(rows, W)
        self.layers = []
        for l in range(L):
            w = torch.zeros(S, H, H)
            for i in range(S):
                e = rows[l][rank * S + i]
                w[i].fill_(-1.0 if e < 0 else e + 10 * l)
            self.layers.append([w])

    def _ep_rank(self):
        return self.rank

    def _ep_maps(self):
        return EngineMaps(self.p2l, self.l2p, self.cnt, num_ranks=R, slots_per_rank=S, num_experts=E)

    def _expert_layers(self):
        return self.layers


def test_vllm_worker_hooks_on_an_eplb_state(monkeypatch):
    """``ConnexEPWorker`` reads vLLM's EplbModelState and EP group."""
    pytest.importorskip("vllm")
    import vllm.distributed
    from connex.ep.vllm_ext import ConnexEPWorker
    rows = [[p % E for p in range(R * S)] for _ in range(L)]
    p2l, l2p, cnt = _vllm_state(rows, 2)
    layers = [_MoELayer([torch.zeros(S, H, H)]) for _ in range(L)]
    model = type("M", (), {"num_logical_experts": E, "moe_layers": layers})()
    ms = type("MS", (), {"physical_to_logical_map": p2l, "logical_to_physical_map": l2p,
                         "logical_replica_count": cnt, "model": model,
                         "expert_load_window": torch.ones(3, L, R * S)})()
    w = ConnexEPWorker()
    w.model_runner = type("MR", (), {"eplb_state": type("ES", (), {"model_states": {"h": ms}})()})()
    monkeypatch.setattr(vllm.distributed, "get_ep_group",
                        lambda: type("G", (), {"rank_in_group": 1, "world_size": R})())
    info = w.connex_ep_info()
    assert (info["ep_rank"], info["num_ranks"], info["slots_per_rank"], info["max_replicas"]) == (1, R, S, 2)
    t = PlacementTable(E, R, S, rows)
    t.mark_down(0)
    t.commit()
    ptr = l2p.data_ptr()
    assert w.connex_ep_apply(json.dumps(t.view()))["applied"]
    assert l2p.data_ptr() == ptr and cnt.tolist() == [[1] * E] * L
    assert l2p[:, :, 0].tolist() == [[4, 5, 6, 7]] * L and (l2p[:, :, 1] == -1).all()
    assert w.connex_ep_load() == [3.0 * L] * (R * S)       # window 3 x L layers


def test_apply_in_place_stale_views_and_width_shrink():
    rows = [[p % E for p in range(R * S)] for _ in range(L)]
    w = _Rank(0, rows, W=3)
    ptrs = [w.l2p.data_ptr(), w.cnt.data_ptr(), w.p2l.data_ptr()]
    t = PlacementTable(E, R, S, rows)
    t.commit()
    assert w.connex_ep_apply(t.view())["applied"]
    assert w.cnt.tolist() == [[2] * E] * L and w.l2p[0, 1, :2].tolist() == [1, 5]
    t.mark_down(1)
    t.commit()
    assert w.connex_ep_apply(json.dumps(t.view()))["epoch"] == t.epoch
    # the column the previous epoch used is cleared in the same copy
    assert (w.l2p[..., 1:] == -1).all() and w.cnt.tolist() == [[1] * E] * L
    assert [w.p2l.data_ptr(), w.cnt.data_ptr()] == [ptrs[2], ptrs[1]] and w.l2p.data_ptr() == ptrs[0]
    assert not w.connex_ep_apply(t.view())["applied"]           # stale / duplicate
    with pytest.raises(ValueError, match="geometry"):
        w.connex_ep_apply(dict(t.view(), epoch=99, num_ranks=3))
    bad = dict(t.view(), epoch=100, routable=[[False] * (R * S)] * L)
    with pytest.raises(ValueError, match="no routable replica"):
        w.connex_ep_apply(bad)


def _collective_rpc_server(workers):
    """vLLM's ``/collective_rpc``: run the method on every worker, one result each."""
    class Handler(BaseHTTPRequestHandler):
        def log_message(self, *a):
            pass

        def do_POST(self):
            req = json.loads(self.rfile.read(int(self.headers["Content-Length"])))
            try:
                out = {"results": [getattr(w, req["method"])(*req["args"]) for w in workers]}
                code = 200
            except Exception as ex:  # noqa: BLE001
                out, code = {"error": repr(ex)}, 500
            data = json.dumps(out).encode()
            self.send_response(code)
            self.send_header("Content-Length", str(len(data)))
            self.end_headers()
            self.wfile.write(data)

    srv = ThreadingHTTPServer(("127.0.0.1", 0), Handler)
    threading.Thread(target=srv.serve_forever, daemon=True).start()
    return srv


def test_controller_migrates_between_two_ranks_over_collective_rpc():
    from connex.ep.vllm_ext import VLLMEPEngine
    rows = [[0, 1, 2, 3, 0, 1, -1, -1] for _ in range(L)]
    ranks = [_Rank(r, rows, W=2) for r in range(R)]
    srv = _collective_rpc_server(ranks)
    try:
        eng = VLLMEPEngine(f"http://127.0.0.1:{srv.server_address[1]}", transport="local", timeout=10)
        table = eng.table()
        assert table.slot_map == rows and table.epoch == 0
        ctl = EPController(table, eng)
        ctl.push(force=True)
        rep = ctl.migrate(2, 6)              # expert 2: slot 2 (rank 0) -> slot 6 (rank 1)
        assert rep["moves"] == L and rep["failed_moves"] == 0 and rep["epoch"] == 2
        for l in range(L):
            assert ranks[1].layers[l][0][2].eq(2 + 10 * l).all()      # the copied weights
            for rk in ranks:
                assert rk.l2p[l, 2].tolist() == [2, 6] and rk.cnt[l].tolist() == [2, 2, 2, 1]
        sums = eng.rpc("connex_ep_checksum", [6])
        assert sums[1] == {"6": float(sum((2 + 10 * l) * H * H for l in range(L)))} and sums[0] == {}
        assert [m["rank"] for m in eng.last["move"]] == [0, 1]
        # a second controller adopts the engine's state and continues its epochs
        t2 = eng.table()
        assert t2.epoch == 2 and t2.slot_map[0][6] == 2
        with pytest.raises(Exception, match="epoch"):
            eng.apply(dict(t2.view(), epoch=1))
    finally:
        srv.shutdown()


# --------------------------------------------------------------- SGLang layout
class FakeMD:
    """The fields of SGLang's ExpertLocationMetadata that the glue writes."""

    def __init__(self, rows, X=3):
        p2l = torch.tensor(rows)
        self.physical_to_logical_map, self.physical_to_logical_map_cpu = p2l.clone(), p2l.clone()
        l2p = torch.full((L, E, X), -1)
        for l in range(L):
            for e in range(E):
                ps = [p for p in range(p2l.shape[1]) if rows[l][p] == e]
                l2p[l, e, :len(ps)] = torch.tensor(ps)
        self.logical_to_all_physical_map, self.logical_to_all_physical_map_cpu = l2p, l2p.clone()
        self.logical_to_all_physical_map_num_valid = (l2p != -1).sum(-1)
        self.logical_to_rank_dispatch_physical_map = None
        self.ep_size, self.num_layers, self.num_logical_experts = R, L, E
        self.num_local_physical_experts = p2l.shape[1] // R


class FakeSGLWorker(sglang_ext.SGLangEPWorker):
    def __init__(self, md, rank, layers):
        self.md, self.rank, self.layers = md, rank, layers

    def _md(self):
        return self.md

    def _ep_rank(self):
        return self.rank

    def _dispatch(self):
        return "dynamic"

    def _expert_layers(self):
        return self.layers


def _linear():
    return [[p % E for p in range(R * S)] for _ in range(L)]


def _pick(md, layer, expert, row):
    """SGLang's dynamic dispatch: replica ``row % num_valid``."""
    n = int(md.logical_to_all_physical_map_num_valid[layer, expert])
    return int(md.logical_to_all_physical_map[layer, expert, row % n])


def test_sglang_apply_writes_metadata_in_place():
    md = FakeMD(_linear())
    ptrs = [md.logical_to_all_physical_map.data_ptr(), md.logical_to_all_physical_map_num_valid.data_ptr()]
    w = FakeSGLWorker(md, 0, [])
    t = PlacementTable(E, R, S, _linear())
    t.mark_down(1)
    t.commit()
    v = t.view()
    assert w.connex_ep_apply(json.dumps(v))["applied"]
    assert ptrs == [md.logical_to_all_physical_map.data_ptr(), md.logical_to_all_physical_map_num_valid.data_ptr()]
    for l in range(L):
        a, c = logical_to_physical(v, l)
        assert md.logical_to_all_physical_map_num_valid[l].tolist() == c == [1] * E
        assert torch.equal(md.logical_to_all_physical_map[l], md.logical_to_all_physical_map_cpu[l])
        for e in range(E):
            assert md.logical_to_all_physical_map[l, e, 0] == a[e][0]
            assert (md.logical_to_all_physical_map[l, e, 1:] == -1).all()
            assert all(_pick(md, l, e, row) // S == 0 for row in range(16))
    assert not w.connex_ep_apply(json.dumps(v))["applied"]
    t.mark_up(1)
    t.commit()
    w.connex_ep_apply(t.view())
    assert md.logical_to_all_physical_map_num_valid.tolist() == [[2] * E] * L
    assert {_pick(md, 0, 1, r) for r in range(4)} == {1, 5}


def test_sglang_static_dispatch_prefers_a_local_replica():
    md = FakeMD(_linear())
    md.logical_to_rank_dispatch_physical_map = torch.zeros(L, E, dtype=torch.long)
    w = FakeSGLWorker(md, 1, [])
    t = PlacementTable(E, R, S, _linear())
    t.commit()
    w.connex_ep_apply(t.view())
    assert md.logical_to_rank_dispatch_physical_map.tolist() == [[4, 5, 6, 7]] * L


class FakeScheduler:
    """The patched scheduler loop: commands queued on rank 0 are pulled with
    the per-iteration aborts and run before the batch."""

    def __init__(self, worker):
        self._connex_ep = worker
        self._connex_ep_q, self._connex_ep_wait = queue.Queue(), {}
        self.stop = False
        self.steps = 0

    def loop(self):
        while not self.stop:
            while not self._connex_ep_q.empty():
                sglang_ext._run_cmd(self, self._connex_ep_q.get_nowait())
            self.steps += 1
            time.sleep(0.001)


def test_sglang_control_endpoint_drives_the_controller():
    from connex.ep.mover import ExpertStore
    from connex.rl.transport import LocalTransport
    W = torch.randn(E, H, H, generator=torch.Generator().manual_seed(0))
    rows = _linear()
    md = FakeMD(rows)
    layers = [[torch.stack([W[rows[l][p]] for p in range(R * S)]).contiguous()] for l in range(L)]
    w = FakeSGLWorker(md, 0, layers)
    w.connex_ep_init = lambda cfg="{}": ExpertStore(0, layers, LocalTransport("sgl-r0")).describe()
    sched = FakeScheduler(w)
    sglang_ext._serve(sched, 0)
    th = threading.Thread(target=sched.loop, daemon=True)
    th.start()
    try:
        eng = sglang_ext.SGLangEPEngine(f"http://127.0.0.1:{sched._connex_ep_srv.server_address[1]}", timeout=10)
        info = eng.info()[0]
        assert (info["num_ranks"], info["slots_per_rank"], info["num_experts"]) == (R, S, E)
        ctl = EPController(eng.table(), eng)
        ctl.push(force=True)
        rep = ctl.drain_rank(1)
        assert rep["uncovered"] == 0 and md.logical_to_all_physical_map_num_valid.tolist() == [[1] * E] * L
        assert eng.last["apply"][0]["applied"] and eng.last["queue_s"]["connex_ep_apply"] >= 0
        with pytest.raises(RuntimeError, match="geometry"):
            eng.rpc("connex_ep_apply", {"epoch": 99, "num_ranks": 9, "slots_per_rank": 1, "slot_map": [[0]]})
        with pytest.raises(RuntimeError, match="not a connex.ep command"):
            eng.rpc("_md")
    finally:
        sched.stop = True
        sched._connex_ep_srv.shutdown()


def test_sglang_init_registers_in_the_background():
    layers = [[torch.zeros(S, H, H)] for _ in range(L)]
    w = FakeSGLWorker(FakeMD(_linear()), 0, layers)
    out = w.connex_ep_init(json.dumps({"transport": "local"}))
    deadline = time.time() + 10
    while out.get("pending") and time.time() < deadline:
        time.sleep(0.01)
        out = w.connex_ep_init(json.dumps({"transport": "local"}))
    assert out["rank"] == 0 and len(out["layers"]) == L
    assert w.connex_ep_init("{}") == out


def test_sglang_control_endpoint_is_advertised(tmp_path, monkeypatch):
    monkeypatch.setenv("CONNEX_EP_CTL_FILE", str(tmp_path / "ctl.json"))
    sched = FakeScheduler(FakeSGLWorker(FakeMD(_linear()), 0, []))
    sched.server_args = type("A", (), {"port": 30000})()
    sglang_ext._serve(sched, 0)
    sglang_ext._advertise(sched)
    th = threading.Thread(target=sched.loop, daemon=True)
    th.start()
    try:
        info = json.load(open(tmp_path / "ctl.json"))
        assert info["server_port"] == 30000 and info["port"] > 0
        eng = sglang_ext.SGLangEPEngine.from_server("http://127.0.0.1:30000", timeout=10)
        assert eng.info()[0]["num_experts"] == E
    finally:
        sched.stop = True
        sched._connex_ep_srv.shutdown()


def _tp_rank_main(rank, port, out):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2)
    try:
        md = FakeMD(_linear())
        sched = FakeScheduler(FakeSGLWorker(md, rank, []))
        if rank != 0:
            del sched._connex_ep_wait
        t = PlacementTable(E, R, S, _linear())
        t.mark_down(1)
        t.commit()
        slot = {"ev": threading.Event(), "res": None}
        if rank == 0:
            sched._connex_ep_wait[7] = slot
        sglang_ext._run_cmd(sched, sglang_ext.ConnexEPCmd(7, "connex_ep_apply", [json.dumps(t.view())]))
        if rank == 0:
            out.put([r["result"]["rank"] for r in slot["res"]] + [slot["ev"].is_set()])
        out.put((rank, md.logical_to_all_physical_map_num_valid.tolist()))
    finally:
        dist.destroy_process_group()


def test_sglang_commands_run_on_every_tp_rank_and_gather():
    import socket
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    procs = [ctx.Process(target=_tp_rank_main, args=(r, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    got = [out.get(timeout=5) for _ in range(3)]
    gathered = [g for g in got if isinstance(g, list)]
    assert gathered == [[0, 1, True]]
    assert sorted(g for g in got if isinstance(g, tuple)) == [(0, [[1] * E] * L), (1, [[1] * E] * L)]
