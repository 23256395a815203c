"""EP control plane, more cases on CPU: a drained rank's unique experts are
copied off it before it stops serving, a move whose source dies mid-copy is
re-planned from another replica, a joining rank gets replicas back, standby
replicas take over without copies, migrations keep standby replicas routed,
an engine that raises during a move leaves no staging slot behind, and a
stale view is ignored by the engine."""
import pytest
import torch

from connex.ep import DOWN, DRAINING, EPController, ExpertStore, LocalEngine, Move, PlacementTable
from connex.rl.transport import LocalTransport

L, H = 2, 4


def _stores(table: PlacementTable, transports=True):
    S = table.slots_per_rank
    stores = []
    for r in range(table.num_ranks):
        layers = []
        for l in range(L):
            w = torch.full((S, H, H), -1.0)
            for i in range(S):
                e = table.slot_map[l][r * S + i]
                if e >= 0:
                    w[i].fill_(e + 100 * l)
            layers.append([w])
        stores.append(ExpertStore(r, layers, LocalTransport(f"epm-{id(table)}-{r}") if transports else None))
    return stores


def _engine(table):
    eng = LocalEngine(_stores(table), table.num_experts)
    eng.loader = lambda layer, expert: [torch.full((H, H), float(expert + 100 * layer))]
    return eng


def _holds(eng, table, slot, layer=0):
    """The expert id the weights in ``slot`` belong to."""
    return int(eng.expert_weight(slot, layer)[0, 0].item()) - 100 * layer


def test_drain_copies_unique_experts_off_the_leaving_rank():
    # rank 1 holds the only copy of experts 2 and 3; ranks 0 and 2 have empty slots
    table = PlacementTable(4, 3, 3, [[0, 1, -1, 2, 3, 0, 1, -1, -1]] * L)
    eng = _engine(table)
    ctl = EPController(table, eng)
    ctl.push(force=True)
    rep = ctl.drain_rank(1)
    assert rep["moves"] == 2 * L and rep["uncovered"] == 0 and rep["failed_moves"] == 0
    assert table.rank_state[1] == DRAINING
    for l in range(L):
        moved = {table.slot_map[l][p] for p in range(9) if table.rank_of(p) != 1}
        assert {2, 3} <= moved
        for p in range(9):
            if table.rank_of(p) != 1 and table.slot_map[l][p] in (2, 3):
                assert _holds(eng, table, p, l) == table.slot_map[l][p]
        # the drained rank routes nothing any more
        assert not any(table.routable_mask(l)[p] for p in table.rank_slots(1))
    x = torch.ones(3, H)
    eng.forward(x, [[2, 3], [0, 1], [3, 0]])         # raises if a token reached a dead / unrouted slot


def test_source_dies_mid_move_is_replanned_from_another_replica():
    # expert 0 lives on ranks 0 and 1; slot 8 (rank 2) will receive it
    table = PlacementTable(3, 3, 3, [[0, 1, -1, 0, 2, -1, 1, 2, -1]] * L)
    eng = _engine(table)
    ctl = EPController(table, eng)
    ctl.push(force=True)
    src0 = table.best_source(0, 0, 8, None)
    real_move = eng.move
    calls = {"n": 0}

    def move(moves, peers, S, loader=None):
        calls["n"] += 1
        if calls["n"] == 1:                          # the chosen source dies while copying
            eng.kill(table.rank_of(src0))
            return [(m, False, "owner unreachable") for m in moves]
        return real_move(moves, peers, S, loader)
    eng.move = move
    rep = ctl.migrate(0, 8)
    assert rep["rounds"] >= 2 and rep["moves"] == L
    assert table.rank_state[table.rank_of(src0)] == DOWN
    for l in range(L):
        assert _holds(eng, table, 8, l) == 0


def test_join_rank_gets_replicas_and_migrate_many():
    table = PlacementTable.spread(4, 3, 3, num_layers=L)
    eng = _engine(table)
    ctl = EPController(table, eng, min_replicas=2)
    ctl.push(force=True)
    ctl.fail_rank(2)
    rep = ctl.join_rank(2, [[-1, -1, -1]] * L)
    assert rep["uncovered"] == 0
    for l in range(L):
        for e in range(4):
            assert len(table.replicas(l, e, live_only=True)) >= 2
    rep = ctl.migrate_many([(0, table.rank_slots(2)[0]), (1, table.rank_slots(2)[1])], layers=[0])
    assert rep["failed_moves"] == 0 and table.slot_map[0][table.rank_slots(2)[0]] == 0


def test_standby_replicas_take_over_without_copies():
    table = PlacementTable(2, 2, 2, [[0, 1, 0, 1]] * L, active_replicas=1)
    eng = _engine(table)
    ctl = EPController(table, eng)
    ctl.push(force=True)
    routed = [p for p in range(4) if table.routable_mask(0)[p]]
    assert len(routed) == 2                           # one active replica per expert
    victim = table.rank_of(routed[0])
    rep = ctl.fail_rank(victim)
    assert rep["moves"] == 0 and rep["uncovered"] == 0
    now = [p for p in range(4) if table.routable_mask(0)[p]]
    assert all(table.rank_of(p) != victim for p in now) and {table.slot_map[0][p] for p in now} == {0, 1}


def test_engine_error_during_a_move_leaves_no_staging_slot():
    table = PlacementTable(2, 2, 3, [[0, 1, -1, 0, 1, -1]] * L)
    eng = _engine(table)
    ctl = EPController(table, eng)
    ctl.push(force=True)

    def boom(*a, **k):
        raise RuntimeError("engine crashed mid-move")
    eng.move = boom
    with pytest.raises(RuntimeError):
        ctl.migrate(1, 2)
    assert not table.staging                           # nothing stays unroutable
    assert eng.view["epoch"] == table.epoch            # the rollback was pushed too


def test_stale_view_is_ignored_and_views_roundtrip():
    table = PlacementTable.linear(4, 2, 3, num_layers=L)
    eng = _engine(table)
    ctl = EPController(table, eng)
    ctl.push(force=True)
    table.mark_down(1)
    ctl.push()
    assert eng.apply(dict(table.view(), epoch=0)) is False
    t2 = PlacementTable.from_dict(table.to_dict())
    assert t2.view() == table.view() and t2.rank_state[1] == DOWN
    assert Move.from_dict(Move(0, 1, 2, 3, -1).to_dict()) == Move(0, 1, 2, 3, -1)
