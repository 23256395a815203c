"""EP control plane on CPU: placement table, repair planning, two-epoch
controller over an in-process group, expert mover, group supervisor."""
import os
import tempfile
import time

import pytest
import torch

from connex.ep.controller import EPController, LocalEngine
from connex.ep.groups import EPGroup, EPGroupSupervisor, pid_alive
from connex.ep.mover import ExpertStore
from connex.ep.placement import (DOWN, DRAINING, UP, Move, PlacementError, PlacementTable, l2p_tensors,
                                 logical_to_physical)


def test_linear_and_spread_layouts():
    t = PlacementTable.linear(8, 2, 5)
    assert t.slot_map[0] == [0, 1, 2, 3, 4, 5, 6, 7, 0, 1]
    s = PlacementTable.spread(4, 2, 4)
    row = s.slot_map[0]
    assert sorted(row) == [0, 0, 1, 1, 2, 2, 3, 3]
    assert all(len({s.rank_of(p) for p, e in enumerate(row) if e == x}) == 2 for x in range(4))
    with pytest.raises(PlacementError):
        PlacementTable.linear(9, 2, 4)


def test_routable_mask_states_and_staging():
    t = PlacementTable.linear(4, 2, 3)   # rank 0: e0 e1 e2, rank 1: e3 e0 e1
    assert all(t.routable_mask(0))
    t.mark_draining(1)
    m = t.routable_mask(0)
    assert m[3] and not m[4] and not m[5]  # draining serves only e3 (no up replica)
    t.mark_down(1)
    assert t.uncovered() == [(0, 3)]
    t.begin_moves([Move(0, 3, 2, None, 2)])
    assert not t.routable_mask(0)[2]
    e0 = t.epoch
    assert t.commit() == e0 + 1 and t.commit() == e0 + 1  # clean -> no bump


def test_active_replicas_limit_and_l2p():
    t = PlacementTable.spread(2, 4, 2, num_layers=2)
    t.active_replicas = 1
    l2p, cnt = logical_to_physical(t.view(), 0)
    assert cnt == [1, 1]
    t.active_replicas = None
    l2p, cnt = logical_to_physical(t.view(), 1)
    assert cnt == [4, 4] and all(len(r) == 4 for r in l2p)
    a, b = l2p_tensors(t.view(), 0, "cpu", max_replicas=8)
    assert a.shape == (2, 8) and a.dtype == torch.int32 and b.tolist() == [4, 4]


def test_plan_repair_prefers_empty_then_most_replicated():
    t = PlacementTable(3, 3, 2, [[0, 1, 2, 0, -1, 0]])
    t.mark_down(1)   # e2 lost (slot 2), e0 keeps slots 0, 5
    moves = t.plan_repair()
    assert len(moves) == 1 and moves[0].expert == 2 and moves[0].dst == 4 and moves[0].src is None
    t2 = PlacementTable(3, 2, 2, [[0, 0, 1, 2]])
    t2.mark_down(1)
    mv = t2.plan_repair()  # one e0 copy may go; the last one may not (best effort)
    assert len(mv) == 1 and mv[0].expert in (1, 2) and mv[0].evicts == 0


def _stores(R, S, L, E, dtype=torch.float32, transport=False):
    from connex.rl.transport import LocalTransport
    stores = []
    for r in range(R):
        layers = []
        for l in range(L):
            w = torch.zeros(S, 4, 4, dtype=dtype)
            for i in range(S):
                w[i].fill_((r * S + i) % E + 100 * l)  # slot p holds expert p % E
            layers.append([w])
        stores.append(ExpertStore(r, layers, LocalTransport(f"ep-r{r}") if transport else None))
    return stores


def test_controller_fail_migrate_and_rejoin_two_epochs():
    R, S, L, E = 4, 4, 2, 8
    table = PlacementTable.linear(E, R, S, num_layers=L)   # slots 8..15 are replicas
    stores = _stores(R, S, L, E, transport=True)   # one-sided host reads between the stores
    eng = LocalEngine(stores, E)
    eng.loader = lambda layer, expert: [torch.full((4, 4), float(expert + 100 * layer))]
    ctl = EPController(table, eng)
    ctl.push(force=True)
    x = torch.ones(6, 4)
    topk = [[0, 3], [1, 2], [7, 5], [4, 6], [3, 3], [0, 7]]
    y0 = eng.forward(x, topk)
    # rank 1 fails: everything it held has a replica on rank 2/3 -> reroute only
    rep = ctl.fail_rank(1)
    # no copy needed: one epoch (route around), the commit epoch adds nothing
    assert rep["uncovered"] == 0 and rep["moves"] == 0 and eng.applied[-1] == rep["epoch"]
    assert torch.allclose(eng.forward(x, topk), y0)
    # slot 12 (rank 3) holds the last live replica of expert 4 (slot 4 is on dead rank 1): refused
    with pytest.raises(PlacementError):
        ctl.migrate(0, 12)
    # expert 5 (live only in slot 13) into slot 2 (expert 2 keeps its replica in slot 10)
    rep = ctl.migrate(5, 2)
    assert rep["moves"] == L and rep["failed_moves"] == 0
    assert eng.expert_weight(2)[0, 0].item() == 5.0
    # a later rejoin with empty slots: repair fills nothing that is already covered
    rep = ctl.join_rank(1, [[-1] * S] * L)
    assert rep["uncovered"] == 0
    assert torch.allclose(eng.forward(x, topk), y0)
    # a stale view is rejected by the engine
    assert eng.apply(dict(table.view(), epoch=0)) is False


def test_move_falls_back_to_checkpoint_when_source_dies():
    R, S, L, E = 2, 2, 1, 3
    table = PlacementTable(E, R, S, [[0, -1, 1, 2]])
    stores = _stores(R, S, L, E)   # no transport between the stores: remote reads fail
    eng = LocalEngine(stores, E)
    eng.loader = lambda layer, expert: [torch.full((4, 4), 42.0)]
    ctl = EPController(table, eng)
    ctl.push(force=True)
    # e2 (slot 3, rank 1) into the empty slot 1 on rank 0: the read fails, the
    # move is re-planned from the checkpoint loader
    rep = ctl.migrate(2, 1)
    assert rep["failed_moves"] == 1 and rep["moves"] == 1 and rep["rounds"] == 2
    assert eng.expert_weight(1)[0, 0].item() == 42.0


def test_expert_store_checksum_and_poison():
    s = _stores(1, 2, 1, 2)[0]
    assert s.checksum(0, 1) == 16.0
    s.poison(0, 1)
    assert torch.isnan(s.layers[0][0][1]).all()


def test_group_supervisor_down_rebuild_rejoin():
    healthy = {"http://g0": True, "http://g1": True}
    with tempfile.TemporaryDirectory() as d:
        f = os.path.join(d, "endpoints")
        restarted = []

        def restart():
            restarted.append(1)
            healthy["http://g1"] = True
            return None

        g0, g1 = EPGroup("g0", "http://g0"), EPGroup("g1", "http://g1", restart=restart)
        sup = EPGroupSupervisor([g0, g1], f, probe_s=0.02, fail_after=2, probe=lambda u: healthy[u])
        assert open(f).read().split() == ["http://g0", "http://g1"]
        healthy["http://g1"] = False
        sup.check_once()
        sup.check_once()
        deadline = time.time() + 3
        while time.time() < deadline and not any(e["kind"] == "rejoin" for e in sup.events):
            time.sleep(0.02)
        kinds = [e["kind"] for e in sup.events]
        assert kinds[:2] == ["down", "rebuild-start"] and "rejoin" in kinds and restarted
        assert open(f).read().split() == ["http://g0", "http://g1"]
        sup.stop()


def test_pid_alive():
    assert pid_alive(os.getpid()) and not pid_alive(2 ** 22 + 12345)
