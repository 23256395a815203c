"""ConnexPPGroup (SGLang ``pp_group`` replacement) driven the way SGLang's PP
scheduler loop drives it: stage 0 sends ``proxy`` steps and receives their
``output`` in launch order, executors receive / answer, a stage without a
request's KV reports it and stage 0 gets the re-prefill call; over the
in-process fake chain and over real endpoints on sockets."""
import threading

import pytest
import torch

from connex.adapters.sglang import MISSING_HERE, MSG_TYPE, REPREFILLED, ConnexPPGroup
from connex.pp.handover import KVLedger
from connex.pp.testing import fake_chain


class Hooks:
    def __init__(self):
        self.ledger, self.released, self.reprefilled, self.aborted = KVLedger(), [], [], []

    def kv_held(self, rid):
        return self.ledger.kv_held(rid)

    def release(self, rids):
        rids = list(rids)
        self.released += rids
        self.ledger.forget(rids)

    def reprefill(self, rids):
        self.reprefilled += list(rids)

    def abort(self, rids):
        self.aborted += list(rids)


def _executor_step(group, hooks):
    td = group.recv_tensor_dict()
    assert td[MSG_TYPE] == "proxy"
    hooks.ledger.commit(td.get("request_ids"), td.get("cx_ctx"), None, td[MISSING_HERE])
    if group.is_last_rank:
        out = {"next_token_ids": (td["hidden_states"] + 1).long()}
    else:
        out = {"hidden_states": td["hidden_states"] + 1, MSG_TYPE: "proxy"}
    group.send_tensor_dict(out)


class Rows:
    rows = (None, None)

    def __call__(self):
        return self.rows


def test_three_stages_two_microbatches_in_launch_order():
    links = fake_chain(3, k=2)
    rows = Rows()
    h = [Hooks() for _ in links]
    g = [ConnexPPGroup(l, hk, row_info=rows if i == 0 else None, recv_timeout_s=1.0)
         for i, (l, hk) in enumerate(zip(links, h))]
    assert g[0].is_first_rank and g[2].is_last_rank and (g[1].prev_rank, g[1].next_rank) == (0, 2)
    rows.rows = (["a"], [0])
    g[0].send_tensor_dict({"hidden_states": torch.zeros(1, 4), MSG_TYPE: "proxy"})
    rows.rows = (["b"], [0])
    g[0].send_tensor_dict({"hidden_states": torch.full((1, 4), 10.0), MSG_TYPE: "proxy"})
    for _ in range(2):
        _executor_step(g[1], h[1])
        _executor_step(g[2], h[2])
    out_a, out_b = g[0].recv_tensor_dict(), g[0].recv_tensor_dict()
    assert out_a[MSG_TYPE] == "output" and out_a["next_token_ids"].tolist() == [[2] * 4]
    assert out_b["next_token_ids"].tolist() == [[12] * 4]
    assert h[1].kv_held("a") == 1 and h[2].kv_held("b") == 1


def test_stage_without_kv_reports_rows_and_stage0_reprefills():
    links = fake_chain(2)
    rows = Rows()
    h0, h1 = Hooks(), Hooks()
    g0 = ConnexPPGroup(links[0], h0, row_info=rows, recv_timeout_s=1.0)
    g1 = ConnexPPGroup(links[1], h1)
    rows.rows = (["r1", "r2"], [5, 0])            # r1 has 5 tokens of context this stage never saw
    g0.send_tensor_dict({"hidden_states": torch.zeros(2, 4)})
    td = g1.recv_tensor_dict()
    assert td[MISSING_HERE] == ["r1"] and "r1" in h1.released
    g1.send_tensor_dict({"next_token_ids": torch.zeros(2, dtype=torch.long), MISSING_HERE: ["ignored"]})
    out = g0.recv_tensor_dict()
    assert out[REPREFILLED] == ["r1"] and h0.reprefilled == ["r1"] and "cx_missing" not in out
    with pytest.raises(RuntimeError):
        g1.send_tensor_dict({})                   # nothing to answer
    with pytest.raises(RuntimeError):
        g0.recv_tensor_dict()                     # nothing outstanding
    with pytest.raises(NotImplementedError):
        g0.send_object({}, 1)


def test_finished_requests_free_kv_downstream():
    links = fake_chain(2)
    rows = Rows()
    h1 = Hooks()
    g0 = ConnexPPGroup(links[0], Hooks(), row_info=rows, recv_timeout_s=1.0)
    g1 = ConnexPPGroup(links[1], h1)
    rows.rows = (["x"], [0])
    g0.send_tensor_dict({"hidden_states": torch.zeros(1, 2)})
    _executor_step(g1, h1)
    g0.recv_tensor_dict()
    g0.finished(["x"])
    rows.rows = (["y"], [0])
    g0.send_tensor_dict({"hidden_states": torch.zeros(1, 2)})
    _executor_step(g1, h1)
    g0.recv_tensor_dict()
    assert h1.released == ["x"] and h1.kv_held("x") == 0 and h1.kv_held("y") == 1


def test_over_real_endpoints():
    from connex.pp.endpoint import PipelineEndpoint
    from connex.pp.routing import StaticMembership
    mem = StaticMembership(0, 0)
    eps = [PipelineEndpoint("m", s, 2, membership=mem, recv_timeout_s=2.0) for s in range(2)]
    for e in eps:
        mem.add(e.stage_idx, 0, e.address)
    h1 = Hooks()
    g0, g1 = ConnexPPGroup(eps[0], Hooks(), recv_timeout_s=2.0), ConnexPPGroup(eps[1], h1)
    stop = threading.Event()

    def serve():
        while not stop.is_set():
            td = g1.try_recv_tensor_dict(0.1)
            if td is not None:
                g1.send_tensor_dict({"next_token_ids": td["hidden_states"].long() + 1})
    t = threading.Thread(target=serve, daemon=True)
    t.start()
    try:
        for i in range(5):
            g0.send_tensor_dict({"hidden_states": torch.full((2, 8), float(i))})
            assert g0.recv_tensor_dict()["next_token_ids"].tolist() == [[i + 1] * 8] * 2
    finally:
        stop.set()
        t.join(2)
        g0.destroy()
        g1.destroy()
