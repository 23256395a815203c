"""Engine-side EP control shared by the vLLM and SGLang glue.

An inference engine keeps the expert placement of an EP deployment in a few
integer tensors that every MoE layer reads on every step:

* ``p2l``   ``[L, P]``    physical slot -> logical expert;
* ``l2p``   ``[L, E, W]`` logical expert -> its physical slots, ``-1`` padded;
* ``count`` ``[L, E]``    replicas per logical expert.

Writing new *contents* into those same tensors between two steps reroutes
every token, also inside captured CUDA graphs (a graph holds the pointers,
not the values).  :class:`EPWorkerCore` implements the RPC surface an
``EPController`` drives (reference ``connex/ep/vllm_ext.py:139-338``,
``connex/ep/sglang_ext.py:286-547``) on top of four engine hooks that the
vLLM and SGLang classes provide:

``_ep_rank()``, ``_ep_maps() -> EngineMaps``, ``_expert_layers()`` (per MoE
layer the expert parameter tensors viewed as ``[local slots, ...]``) and,
optionally, ``_ep_order_writes(stream)`` (make the map writes wait for work
on other streams that may still read the old maps).

How the map update runs on the device: the new contents (a few KB) are built
on the host in pinned memory and copied with ``non_blocking=True`` on the
engine's current stream, so the next forward is ordered after the writes
without the host waiting for the GPU.  An event recorded after the copies
keeps the pinned buffers alive until they are consumed, and an expert move
into slots that an epoch has just staged out starts only after that event
(earlier batches may still read those slots).  ``CONNEX_EP_APPLY_SYNC=1``
selects a blocking variant that synchronises the device around the writes.

Expert weights move through :class:`connex.ep.mover.ExpertStore`: inside an
NVLink box one ``copy_segments`` launch per source rank reads the rows over
CUDA IPC mappings on a low-priority stream while the engine keeps serving.

:class:`HTTPEPEngine` is the controller-side handle (``apply`` / ``describe``
/ ``move`` / ``info`` / ``table`` / ``load``) over an engine's RPC endpoint;
the vLLM and SGLang modules subclass it for their endpoints.
"""
from __future__ import annotations

import json
import logging
import os
import threading
import time
import urllib.error
import urllib.request
from dataclasses import dataclass
from typing import Any, List, Optional

log = logging.getLogger("connex.ep")


def _arg(x):
    """RPC arguments arrive as JSON strings over HTTP, as objects in-process."""
    return json.loads(x) if isinstance(x, str) else x


def slot_sums(layers, slots, slots_per_rank: int, budget: int = 64 << 20) -> dict:
    """``{str(global slot): float64 sum of that slot over every layer and
    parameter}`` for the given global slots of one rank.

    The sums stay on the device until one copy back at the end; slots are
    gathered in chunks so that the float64 transient of one chunk stays under
    ``budget`` bytes (a whole rank's experts in float64 would be GBs)."""
    import torch
    slots = list(slots)
    if not slots:
        return {}
    acc = None
    for params in layers:
        for w in params:
            per_slot = max(1, w[0].numel() * 8)
            step = max(1, budget // per_slot)
            parts = []
            for j in range(0, len(slots), step):
                idx = torch.tensor([p % slots_per_rank for p in slots[j:j + step]], device=w.device)
                parts.append(w.index_select(0, idx).reshape(len(idx), -1).double().sum(dim=1))
            s = parts[0] if len(parts) == 1 else torch.cat(parts)
            acc = s if acc is None else acc + s.to(acc.device)
    return {str(p): float(v) for p, v in zip(slots, acc.tolist())}


@dataclass
class EngineMaps:
    """The placement tensors of one engine process (device or host)."""
    p2l: Any                      # [L, P]
    l2p: Any                      # [L, E, W]
    count: Any                    # [L, E]
    num_ranks: int
    slots_per_rank: int
    num_experts: int
    p2l_cpu: Any = None           # host mirrors some engines keep next to the device maps
    l2p_cpu: Any = None
    rank_pick: Any = None         # [L, E] static dispatch: the slot this rank sends an expert to
    dispatch: str = "dynamic"

    @property
    def num_layers(self) -> int:
        return int(self.p2l.shape[0])

    @property
    def width(self) -> int:
        return int(self.l2p.shape[-1])


def build_maps(view: dict, maps: EngineMaps, rank: int, prev_width: int):
    """Host contents for ``maps`` from a ``PlacementTable.view()``:
    ``(rows [L][P], l2p [L, E, w'], count [L, E], rank_pick or None, w)``
    where ``w`` is the widest replica list and ``w' = max(w, prev_width)``
    (columns a previous epoch used are rewritten with -1 in the same copy)."""
    import torch
    from connex.ep.placement import logical_to_physical
    if view["num_ranks"] != maps.num_ranks or view["slots_per_rank"] != maps.slots_per_rank:
        raise ValueError(f"view geometry {view['num_ranks']}x{view['slots_per_rank']} != engine "
                         f"{maps.num_ranks}x{maps.slots_per_rank}")
    L = maps.num_layers
    nl = len(view["slot_map"])
    if nl not in (1, L):
        raise ValueError(f"view has {nl} layers, engine {L}")
    per_layer = []
    for layer in range(nl):
        lists, cnt = logical_to_physical(view, layer)
        if min(cnt) == 0:
            raise ValueError(f"layer {layer}: an expert has no routable replica")
        per_layer.append(([[p for p in ps if p >= 0] for ps in lists], cnt))
    w = max(max(c) for _, c in per_layer)
    if w > maps.width:
        raise ValueError(f"{w} replicas per expert, engine allows {maps.width}")
    if nl != L:
        per_layer = per_layer * L
    rows = view["slot_map"] if nl == L else view["slot_map"] * L
    cols = min(maps.width, max(w, prev_width))
    l2p = torch.full((L, maps.num_experts, cols), -1, dtype=maps.l2p.dtype)
    cnt = torch.empty((L, maps.num_experts), dtype=maps.count.dtype)
    pick = None
    if maps.rank_pick is not None:
        pick = torch.empty(tuple(maps.rank_pick.shape), dtype=maps.rank_pick.dtype)
    S = maps.slots_per_rank
    for l, (lists, c) in enumerate(per_layer):
        cnt[l] = torch.tensor(c, dtype=cnt.dtype)
        for e, ps in enumerate(lists):
            l2p[l, e, :len(ps)] = torch.tensor(ps, dtype=l2p.dtype)
            if pick is not None:
                pick[l, e] = next((p for p in ps if p // S == rank), ps[0])
    return rows, l2p, cnt, pick, w


class EPWorkerCore:
    """The ``connex_ep_*`` RPCs; mixed into an engine's worker / scheduler
    object.  State lives in ``_cx_*`` attributes created on first use (the
    vLLM worker extension is mixed into a class whose ``__init__`` is not
    ours)."""

    # ---- engine hooks -------------------------------------------------------
    def _ep_rank(self) -> int:
        raise NotImplementedError

    def _ep_maps(self) -> EngineMaps:
        raise NotImplementedError

    def _expert_layers(self) -> list:
        raise NotImplementedError

    def _ep_order_writes(self, stream) -> None:
        """Order the map writes after other streams that read the maps."""

    def _ep_load_counts(self):
        return None

    # ---- state ------------------------------------------------------------
    def _cx(self) -> dict:
        st = self.__dict__.get("_cx_state")
        if st is None:
            st = self.__dict__["_cx_state"] = {"epoch": 0, "rows": None, "width": None, "store": None,
                                                "init_job": None, "move_job": None, "written": None,
                                                "lock": threading.Lock()}
        return st

    # ---- RPCs --------------------------------------------------------------
    def connex_ep_info(self):
        m = self._ep_maps()
        rows = m.p2l_cpu if m.p2l_cpu is not None else m.p2l
        return {"ep_rank": self._ep_rank(), "num_ranks": m.num_ranks, "slots_per_rank": m.slots_per_rank,
                "num_layers": m.num_layers, "num_experts": m.num_experts, "max_replicas": m.width,
                "slot_map": rows.cpu().tolist(), "dispatch": m.dispatch, "epoch": self._cx()["epoch"]}

    def _make_transport(self, cfg: dict):
        kind = cfg.get("transport", "ipc")
        if kind in ("ipc", "none", None):
            return None                   # same-box peers read through CUDA IPC only
        from connex.rl.transport import make_transport
        alias = {"connex-rs": "engine", "cxengine": "engine"}
        return make_transport(alias.get(kind, kind), name=f"ep-r{self._ep_rank()}-g{int(cfg.get('group', 0))}")

    def connex_ep_init(self, cfg="{}"):
        """Expose this rank's expert weights to its peers.  Registration (IPC
        export, transport registration) runs in a background thread so the
        engine keeps stepping; the call returns ``{"pending": True}`` until it
        is done, then ``ExpertStore.describe()``.  Call again to poll."""
        cfg = _arg(cfg) or {}
        st = self._cx()
        if st["store"] is not None:
            return st["store"].describe()
        job = st["init_job"]
        if job is None:
            from connex.ep.mover import ExpertStore
            layers, rank = self._expert_layers(), self._ep_rank()
            job = st["init_job"] = {"done": False, "error": None}

            def run():
                try:
                    dev = layers[0][0].device if layers else None
                    if dev is not None and dev.type == "cuda":
                        import torch
                        torch.cuda.set_device(dev)
                    t0 = time.perf_counter()
                    store = ExpertStore(rank, layers, self._make_transport(cfg))
                    job["describe"] = store.describe()
                    st["store"] = store
                    log.info("connex.ep rank %d: experts registered in %.0f ms", rank,
                             (time.perf_counter() - t0) * 1e3)
                except Exception as ex:  # noqa: BLE001
                    job["error"] = repr(ex)
                job["done"] = True

            threading.Thread(target=run, daemon=True, name="connex-ep-init").start()
        if not job["done"]:
            return {"pending": True, "rank": self._ep_rank()}
        if job["error"]:
            st["init_job"] = None              # the caller may retry
            raise RuntimeError(job["error"])
        return job["describe"]

    def connex_ep_apply(self, view):
        import torch
        t0 = time.perf_counter()
        view = _arg(view)
        st = self._cx()
        if view["epoch"] <= st["epoch"] and st["epoch"] > 0:
            return {"applied": False, "epoch": st["epoch"]}
        m = self._ep_maps()
        prev_w = st["width"] if st["width"] is not None else m.width
        rows, l2p, cnt, pick, w = build_maps(view, m, self._ep_rank(), prev_w)
        rows_t = None if rows == st["rows"] else torch.tensor(rows, dtype=m.p2l.dtype)
        dev = m.l2p.device
        if dev.type != "cuda":
            self._write(m, rows_t, l2p, cnt, pick, False)
        elif os.environ.get("CONNEX_EP_APPLY_SYNC", "0") == "1":
            torch.cuda.synchronize(dev)
            self._write(m, rows_t, l2p, cnt, pick, False)
            torch.cuda.synchronize(dev)
        else:
            stream = torch.cuda.current_stream(dev)
            self._ep_order_writes(stream)
            staged = [x.pin_memory() for x in (rows_t, l2p, cnt, pick) if x is not None]
            it = iter(staged)
            pinned = [next(it) if x is not None else None for x in (rows_t, l2p, cnt, pick)]
            self._write(m, pinned[0], pinned[1], pinned[2], pinned[3], True)
            ev = torch.cuda.Event()
            ev.record(stream)
            st["written"] = (ev, staged)      # buffers live until the copies ran
        if rows_t is not None:
            st["rows"] = rows
        st["width"] = w
        st["epoch"] = view["epoch"]
        return {"applied": True, "epoch": view["epoch"], "rank": self._ep_rank(),
                "apply_ms": (time.perf_counter() - t0) * 1e3}

    @staticmethod
    def _write(m: EngineMaps, rows, l2p, cnt, pick, non_blocking: bool) -> None:
        dev = m.l2p.device
        cols = l2p.shape[-1]
        if rows is not None:
            m.p2l.copy_(rows.to(dev, non_blocking=non_blocking))
            if m.p2l_cpu is not None:
                m.p2l_cpu.copy_(rows)
        m.l2p[..., :cols].copy_(l2p.to(dev, non_blocking=non_blocking))
        if m.l2p_cpu is not None:
            m.l2p_cpu[..., :cols].copy_(l2p)
        m.count.copy_(cnt.to(dev, non_blocking=non_blocking))
        if pick is not None:
            m.rank_pick.copy_(pick.to(dev, non_blocking=non_blocking))

    def _store(self):
        s = self._cx()["store"]
        if s is None:
            raise RuntimeError("call connex_ep_init first")
        return s

    def _before_move(self) -> None:
        """Moves may overwrite slots the last epoch staged out: wait until
        the batches that could still read them (everything queued before the
        map writes) have finished."""
        w = self._cx()["written"]
        if w is not None:
            w[0].synchronize()

    def _run_moves(self, req: dict):
        from connex.ep.placement import Move
        moves = [Move.from_dict(x) for x in req["moves"]]
        peers = {int(k): v for k, v in req["peers"].items()}
        self._before_move()
        res = self._store().apply_moves(moves, peers, req["slots_per_rank"], timeout_ms=req.get("timeout_ms"))
        return [[mv.to_dict(), ok, err] for mv, ok, err in res]

    def connex_ep_move(self, req):
        req = _arg(req)
        t0 = time.perf_counter()
        results = self._run_moves(req)
        return {"rank": self._ep_rank(), "seconds": time.perf_counter() - t0, "results": results}

    def connex_ep_move_start(self, req):
        """Start the moves in a background thread and return at once: the
        engine keeps stepping while the weights move.  Poll with
        ``connex_ep_move_poll``."""
        req = _arg(req)
        st = self._cx()
        store = self._store()
        with st["lock"]:
            prev = st["move_job"]
            if prev is not None and not prev["done"]:
                raise RuntimeError("a move is already running")
            job = st["move_job"] = {"done": False, "results": [], "seconds": None, "error": None}

        def run():
            t0 = time.perf_counter()
            try:
                dev = store.layers[0][0].device if store.layers else None
                if dev is not None and dev.type == "cuda":
                    import torch
                    torch.cuda.set_device(dev)
                job["results"] = self._run_moves(req)
            except Exception as ex:  # noqa: BLE001
                job["error"] = repr(ex)
            job["seconds"] = time.perf_counter() - t0
            job["done"] = True

        threading.Thread(target=run, daemon=True, name="connex-ep-move").start()
        return {"rank": self._ep_rank(), "started": True}

    def connex_ep_move_poll(self):
        job = self._cx()["move_job"]
        if job is None:
            return {"rank": self._ep_rank(), "done": True, "results": [], "seconds": 0.0, "error": None}
        return {"rank": self._ep_rank(), **job}

    def _mine(self, slots):
        m = self._ep_maps()
        S, rank = m.slots_per_rank, self._ep_rank()
        want = slots or range(rank * S, (rank + 1) * S)
        return [p for p in want if p // S == rank], S

    def connex_ep_checksum(self, slots="[]"):
        """float64 sum per local slot over every MoE layer (all local slots
        when ``slots`` is empty).  Verification helper."""
        mine, S = self._mine(_arg(slots))
        return slot_sums(self._expert_layers(), mine, S)

    def connex_ep_poison(self, slots="[]", value="nan"):
        """Fill the given global slots of this rank with ``value`` (tests:
        shows that no token reaches them)."""
        import torch
        m = self._ep_maps()
        S, rank = m.slots_per_rank, self._ep_rank()
        mine = [p for p in (_arg(slots) or []) if p // S == rank]
        for p in mine:
            for params in self._expert_layers():
                for w in params:
                    w[p % S].fill_(float(value))
        if torch.cuda.is_available():
            torch.cuda.synchronize()
        return len(mine)

    def connex_ep_load(self):
        return self._ep_load_counts()


class HTTPEPEngine:
    """``EPController`` engine handle for one engine server (all its EP
    ranks) over an HTTP RPC endpoint: POST ``{"method", "args", "timeout"}``,
    one result per rank.  Subclasses set :attr:`path` and unwrap results."""

    path = "/rpc"

    def __init__(self, base_url: str, transport: str = "ipc", group: int = 0, timeout: float = 120.0,
                 async_moves: bool = True, poll_s: float = 0.005):
        self.base = base_url.rstrip("/")
        self.cfg = {"transport": transport, "group": group}
        self.timeout = timeout
        self.async_moves = async_moves
        self.poll_s = poll_s
        self.last: dict = {}
        self._opener = urllib.request.build_opener(urllib.request.ProxyHandler({}))

    def _post(self, method: str, args) -> tuple:
        body = json.dumps({"method": method, "timeout": self.timeout,
                           "args": [a if isinstance(a, str) else json.dumps(a) for a in args]}).encode()
        req = urllib.request.Request(self.base + self.path, data=body, method="POST",
                                     headers={"Content-Type": "application/json"})
        try:
            with self._opener.open(req, timeout=self.timeout + 5) as r:
                return r.status, json.loads(r.read())
        except urllib.error.HTTPError as e:
            return e.code, e.read().decode(errors="replace")

    def _unwrap(self, method: str, body) -> List[Any]:
        return body.get("results", body) if isinstance(body, dict) else body

    def rpc(self, method: str, *args) -> List[Any]:
        status, body = self._post(method, args)
        if status != 200:
            raise RuntimeError(f"{method}: HTTP {status} {str(body)[:300]}")
        return self._unwrap(method, body)

    def info(self):
        return self.rpc("connex_ep_info")

    def table(self):
        """The placement the engine runs now, at its epoch (a new controller
        continues the epoch sequence from there)."""
        from connex.ep.placement import PlacementTable
        infos = self.info()
        i = infos[0]
        return PlacementTable(i["num_experts"], i["num_ranks"], i["slots_per_rank"], i["slot_map"],
                              epoch=max(x["epoch"] for x in infos))

    def describe(self) -> dict:
        """Every rank's ``ExpertStore.describe()`` (registration runs in the
        background on the ranks: poll until all are ready)."""
        deadline = time.time() + self.timeout
        while True:
            res = self.rpc("connex_ep_init", self.cfg)
            if not any(isinstance(d, dict) and d.get("pending") for d in res):
                return {d["rank"]: d for d in res}
            if time.time() > deadline:
                raise TimeoutError("connex_ep_init still pending")
            time.sleep(0.02)

    def apply(self, view: dict):
        res = self.rpc("connex_ep_apply", view)
        self.last["apply"] = res
        newer = [r["epoch"] for r in res if not r.get("applied") and r["epoch"] > view["epoch"]]
        if newer:
            from connex.ep.placement import PlacementError
            raise PlacementError(f"engine runs epoch {max(newer)} > {view['epoch']}: another controller "
                                 "owns it (adopt its state with table())")
        return res

    def move(self, moves, peers: dict, slots_per_rank: int):
        from connex.ep.placement import Move
        req = {"moves": [m.to_dict() for m in moves], "peers": {str(k): v for k, v in peers.items()},
               "slots_per_rank": slots_per_rank}
        if self.async_moves:
            self.rpc("connex_ep_move_start", req)
            deadline = time.time() + self.timeout
            while True:
                res = self.rpc("connex_ep_move_poll")
                if all(r["done"] for r in res):
                    break
                if time.time() > deadline:
                    raise TimeoutError("expert moves still running")
                time.sleep(self.poll_s)
            errs = [r["error"] for r in res if r.get("error")]
            if errs:
                raise RuntimeError(f"expert move failed: {errs}")
        else:
            res = self.rpc("connex_ep_move", req)
        self.last["move"] = [{"rank": r["rank"], "seconds": r["seconds"]} for r in res]
        return [(Move.from_dict(m), ok, err) for r in res for m, ok, err in r["results"]]

    def load(self):
        return self.rpc("connex_ep_load")


__all__ = ["EngineMaps", "EPWorkerCore", "HTTPEPEngine", "build_maps", "slot_sums"]
