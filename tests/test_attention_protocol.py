"""Barrier protocol of the persistent two-tile prefill attention, checked on
the CPU.  ``prefill_attn_pair_kernel`` (``connex_b200/csrc/kernels/
attention_tc.cu``) runs three kinds of roles over mbarriers: one TMA producer
thread, one MMA thread and two softmax warpgroups (one per 128-row Q tile).
An mbarrier wait only sees the *parity* of the phase it waits for, so a
barrier that completes two phases before its waiter looks at it is
indistinguishable from one that completed none.  This model replays the
roles' waits, arrivals and commits in the kernel's order, with TMA loads and
tensor-core commits landing after random delays and the roles interleaved at
random, over random work items, and checks that

* every role finishes (no lost arrival, no circular wait);
* no successful wait finds its barrier more than one phase past the phase it
  waited for (so the parity test is exact);
* for each Q tile the tensor core runs every P.V before the next Q.K^T that
  overwrites the same tensor-memory columns, and each softmax step sees
  exactly the scores it waited for.

A negative control replays the rejected design that signals "O final" on
the scores barrier: there the persistent MMA thread can commit the next
item's first scores before the softmax has waited for O, and the model must
catch it.
"""
import random

import pytest


class Bar:
    """An mbarrier: ``count`` arrivals complete a phase."""

    def __init__(self, name, count=1):
        self.name, self.count, self.pending, self.done = name, count, 0, 0

    def arrive(self):
        self.pending += 1
        if self.pending == self.count:
            self.pending = 0
            self.done += 1


class Model:
    def __init__(self, items, rng, o_final_on_s=False):
        self.rng = rng
        self.o_final_on_s = o_final_on_s      # the rejected design (negative control)
        self.partial_tail = {i for i in range(len(items)) if rng.random() < 0.5}   # paged items
        self.items = items
        b = {}
        for x in range(2):
            for n in ("q_full", "q_empty", "k_full", "k_empty", "v_full", "v_empty", "s_full", "o_full"):
                b[f"{n}{x}"] = Bar(f"{n}{x}")
            b[f"p_full{x}"] = Bar(f"p_full{x}", count=1)   # the warpgroup's 128 arrivals, as one
        self.b = b
        self.async_q = []            # (deadline, callback): TMA completions
        self.mma_q = []              # tensor-core work in issue order: (op, tag)
        self.clock = 0
        self.qk_exec = [0, 0]        # Q_x.K^T executed so far (each overwrites S_x)
        self.pv_exec = [0, 0]        # P_x.V executed so far (each reads P_x from S_x's columns)
        self.errors = []

    # --- asynchronous engines --------------------------------------------
    def tma(self, bar):
        self.async_q.append((self.clock + self.rng.randint(1, 6), bar.arrive))

    def mma(self, op, tag):
        self.mma_q.append((op, tag))

    def step_engines(self):
        ready = [e for e in self.async_q if e[0] <= self.clock]
        for e in ready:
            self.async_q.remove(e)
            e[1]()
        if self.mma_q and self.rng.random() < 0.5:     # the tensor core retires one op, in order
            op, tag = self.mma_q.pop(0)
            if op == "qk":
                x = tag[0]
                if self.pv_exec[x] < self.qk_exec[x]:     # the P held in S_x not read yet
                    self.errors.append(f"Q{x}.K^T #{self.qk_exec[x]} overwrote S_{x} before its P.V ran")
                self.qk_exec[x] += 1
            elif op == "pv":
                self.pv_exec[tag[0]] += 1
            elif op == "commit":
                tag.arrive()

    # --- role helpers -----------------------------------------------------
    def wait(self, bar, phase):
        """Generator: wait for phase ``phase`` (0-based count) of ``bar``."""
        while True:
            if (bar.done & 1) != (phase & 1) and bar.done >= phase + 1:
                if bar.done > phase + 1:
                    self.errors.append(f"{bar.name}: waited for phase {phase}, found {bar.done} done")
                return
            if (bar.done & 1) != (phase & 1) and bar.done < phase + 1:
                self.errors.append(f"{bar.name}: parity says phase {phase} done but only {bar.done} are")
                return
            yield

    # --- the kernel's roles ------------------------------------------------
    def producer(self):
        kv = 0
        nk, nv = [0, 0], [0, 0]
        for n_it, (nt, nkv) in enumerate(self.items):
            for x in range(2):
                yield from self.wait(self.b[f"q_empty{x}"], n_it - 1) if n_it else iter(())
                self.tma(self.b[f"q_full{x}"])
            def load(kind, j):
                u = kv + j
                s = u & 1
                cnt = nk if kind == "k" else nv
                if cnt[s]:
                    yield from self.wait(self.b[f"{kind}_empty{s}"], cnt[s] - 1)
                cnt[s] += 1
                self.tma(self.b[f"{kind}_full{s}"])
            for j in range(nkv):
                yield from load("k", j)
                if j >= 1:
                    yield from load("v", j - 1)
            if nkv:
                yield from load("v", nkv - 1)
            kv += nkv

    def mma_thread(self):
        kv = 0
        pf = [0, 0]
        def commit(name):
            self.mma("commit", self.b[name])
        def wait_k(u):
            s = u & 1
            yield from self.wait(self.b[f"k_full{s}"], u >> 1)
        for n_it, (nt, nkv) in enumerate(self.items):
            for x in range(2):
                yield from self.wait(self.b[f"q_full{x}"], n_it)
            yield from wait_k(kv)
            for x in range(2):
                if nt[x] == 0:
                    continue
                self.mma("qk", (x, 0))
                commit(f"s_full{x}")
                if nt[x] == 1:
                    commit(f"q_empty{x}")
            commit(f"k_empty{kv & 1}")
            for j in range(nkv):
                u = kv + j
                s = u & 1
                yield from self.wait(self.b[f"v_full{s}"], u >> 1)
                for x in range(2):
                    if j >= nt[x]:
                        continue
                    yield from self.wait(self.b[f"p_full{x}"], pf[x])
                    pf[x] += 1
                    self.mma("pv", (x, j))
                    if j + 1 < nt[x]:
                        yield from wait_k(u + 1)
                        self.mma("qk", (x, j + 1))
                        commit(f"s_full{x}")
                        if j + 2 == nt[x]:
                            commit(f"q_empty{x}")
                    else:
                        commit(f"s_full{x}" if self.o_final_on_s else f"o_full{x}")
                commit(f"v_empty{s}")
                if j + 1 < nkv:
                    commit(f"k_empty{(u + 1) & 1}")
            for x in range(2):
                if nt[x] == 0:
                    commit(f"q_empty{x}")
            kv += nkv

    def softmax(self, x):
        sw = ow = steps = 0          # phases waited on s_full / o_full; score steps taken
        kv = 0                       # ring position of the item's key tile 0
        for n_it, (nt, nkv) in enumerate(self.items):
            zero_x = 0 if nt[0] == nkv else 1     # the tile whose P.V reads the last V tile first
            for j in range(nt[x]):
                yield from self.wait(self.b[f"s_full{x}"], sw)
                sw += 1
                steps += 1
                if self.qk_exec[x] != steps:       # exactly the scores this step waited for
                    self.errors.append(f"softmax {x} step {steps - 1} saw {self.qk_exec[x]} Q.K^T done")
                yield                                   # compute
                if x == zero_x and j == nkv - 1 and n_it in self.partial_tail:
                    # paged: unwritten cache rows of the last V tile are zeroed
                    # before this tile's P.V (a second consumer of v_full)
                    u = kv + j
                    yield from self.wait(self.b[f"v_full{u & 1}"], u >> 1)
                self.b[f"p_full{x}"].arrive()
            if nt[x]:
                if self.o_final_on_s:
                    yield from self.wait(self.b[f"s_full{x}"], sw)
                    sw += 1
                else:
                    yield from self.wait(self.b[f"o_full{x}"], ow)
                    ow += 1
                yield                                   # epilogue
            kv += nkv

    def run(self, max_steps=200000):
        roles = [self.producer(), self.mma_thread(), self.softmax(0), self.softmax(1)]
        live = list(roles)
        for _ in range(max_steps):
            self.clock += 1
            self.step_engines()
            if not live:
                return True
            r = self.rng.choice(live)
            try:
                next(r)
            except StopIteration:
                live.remove(r)
        return False


def _items(rng, n):
    """Random work items: (key tiles of Q tile 0 and 1, key tiles loaded).
    Tile 1 takes part in the same tiles plus at most one more, or none (it
    lies past the sequence end), as ``item_of`` in the kernel computes."""
    out = []
    for _ in range(n):
        n0 = rng.randint(1, 6)
        r = rng.random()
        n1 = 0 if r < 0.2 else (n0 if r < 0.5 else n0 + 1)
        out.append(((n0, n1), max(n0, n1)))
    return out


@pytest.mark.parametrize("seed", range(40))
def test_barrier_protocol_has_no_lost_phase_and_no_deadlock(seed):
    rng = random.Random(seed)
    m = Model(_items(rng, rng.randint(1, 6)), rng)
    finished = m.run()
    assert finished, "a role is still waiting: lost arrival or circular wait"
    assert m.errors == []
    assert m.qk_exec == m.pv_exec == [sum(nt[x] for nt, _ in m.items) for x in range(2)]


def test_the_model_catches_o_final_on_the_scores_barrier():
    """The rejected design: with O-final committed on s_full, some schedule
    finds s_full two phases ahead (or deadlocks)."""
    caught = 0
    for seed in range(60):
        rng = random.Random(1000 + seed)
        items = [((n, n), n) for n in (rng.randint(1, 3) for _ in range(4))]
        m = Model(items, rng, o_final_on_s=True)
        finished = m.run(max_steps=20000)
        caught += (not finished) or bool(m.errors)
    assert caught > 0
