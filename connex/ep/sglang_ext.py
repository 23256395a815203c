"""SGLang glue for ``connex.ep`` (upstream SGLang, no fork; the scheduler,
``ExpertLocationMetadata`` and ``TopK`` interfaces of SGLang 0.5).

SGLang keeps an EP deployment's placement in one ``ExpertLocationMetadata``
per process: ``physical_to_logical_map [L, P]``,
``logical_to_all_physical_map [L, E, X]`` (-1 padded),
``logical_to_all_physical_map_num_valid [L, E]``, host mirrors of the first
two, and for static dispatch ``logical_to_rank_dispatch_physical_map``.  The
MoE top-k reads them through ``ExpertLocationDispatchInfo`` (dynamic dispatch
picks replica ``row % num_valid``), so rewriting their contents reroutes
tokens, inside captured CUDA graphs too (reference
``connex/ep/sglang_ext.py:1-44``).

Control path.  The ``connex_ep`` ``sglang.srt.plugins`` entry point (opt-in
with ``CONNEX_EP=1``) patches the scheduler: TP rank 0 serves a small HTTP
endpoint (``CONNEX_EP_PORT``, default any free port, advertised in
:func:`ctl_file`).  A posted command is queued and handed to SGLang's
per-iteration request broadcast (the one that carries timeout aborts), so
every TP rank runs it between the same two forward steps; the per-rank
results are gathered over the TP CPU group and rank 0 answers.  The commands
are :class:`connex.ep.engine_ext.EPWorkerCore`'s ``connex_ep_*`` RPCs.

Serving needs ``--ep-num-redundant-experts`` (room for replicas),
``--ep-dispatch-algorithm dynamic`` (or static) and a model with SGLang EPLB
support; ``--enable-eplb`` stays off (Connex owns the map).  With the overlap
scheduler the previous batch may still run on the forward stream, so the map
writes are ordered after it on the device (the scheduler stream waits for the
forward stream; the next forward waits for the scheduler stream).

Controller side: :class:`SGLangEPEngine`.
"""
from __future__ import annotations

import json
import logging
import os
import queue
import tempfile
import threading
import time
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer

from connex.ep.engine_ext import EngineMaps, EPWorkerCore, HTTPEPEngine

log = logging.getLogger("connex.ep")

_installed = False


class ConnexEPCmd:
    """One control command, carried by SGLang's per-iteration request broadcast."""

    def __init__(self, seq: int, method: str, args):
        self.seq = seq
        self.method = method
        self.args = list(args)
        self.t_enq = time.time()


def register() -> None:
    """``sglang.srt.plugins`` entry point; opt-in with ``CONNEX_EP=1``."""
    if os.environ.get("CONNEX_EP", "").lower() not in ("1", "true", "yes"):
        return
    try:
        install()
    except ImportError as ex:
        log.warning("connex.ep: SGLang scheduler not patched (%s)", ex)


def install() -> None:
    """Patch SGLang's scheduler with the control path (idempotent)."""
    global _installed
    if _installed:
        return
    from sglang.srt.managers.scheduler import Scheduler
    _installed = True
    init0, poll0, process0 = Scheduler.__init__, Scheduler._poll_timeout_aborts, Scheduler.process_input_requests

    def __init__(self, *a, **kw):
        init0(self, *a, **kw)
        try:
            _setup(self)
        except Exception:  # noqa: BLE001  (the server must come up regardless)
            log.exception("connex.ep: control endpoint not started")

    def _poll_timeout_aborts(self):
        out = poll0(self)
        q = getattr(self, "_connex_ep_q", None)
        if q is None or q.empty():
            return out
        out = list(out)
        while True:
            try:
                out.append(q.get_nowait())
            except queue.Empty:
                return out

    def process_input_requests(self, recv_reqs):
        cmds = [r for r in recv_reqs or () if isinstance(r, ConnexEPCmd)]
        if cmds:
            for c in cmds:
                _run_cmd(self, c)
            recv_reqs = [r for r in recv_reqs if not isinstance(r, ConnexEPCmd)]
        return process0(self, recv_reqs)

    Scheduler.__init__ = __init__
    Scheduler._poll_timeout_aborts = _poll_timeout_aborts
    Scheduler.process_input_requests = process_input_requests
    _patch_topk()


def _patch_topk() -> None:
    """Make every MoE path route through the location metadata.  Some models
    call ``TopK`` without ``expert_location_dispatch_info`` on their
    non-all-to-all path, and their logical ids are then used as slot ids:
    replicas are never used.  ``TopK`` knows its layer id, so the dispatch
    info is built from it when the caller passed none."""
    from sglang.srt.layers.moe.topk import TopK
    fwd0 = TopK.forward_cuda
    if getattr(fwd0, "_connex_ep", False):
        return

    def forward_cuda(self, hidden_states, router_logits, *a, **kw):
        layer = getattr(self, "layer_id", None)
        if kw.get("expert_location_dispatch_info") is None and layer is not None:
            from sglang.srt.eplb.expert_location import get_global_expert_location_metadata
            from sglang.srt.eplb.expert_location_dispatch import ExpertLocationDispatchInfo
            md = get_global_expert_location_metadata()
            if md is not None and layer < md.num_layers:
                kw["expert_location_dispatch_info"] = ExpertLocationDispatchInfo.init_new(layer_id=layer)
        return fwd0(self, hidden_states, router_logits, *a, **kw)

    forward_cuda._connex_ep = True
    TopK.forward_cuda = forward_cuda


def _tp_rank() -> int:
    from sglang.srt.runtime_context import get_parallel
    return get_parallel().tp_rank


def _setup(sched) -> None:
    sched._connex_ep = SGLangEPWorker(sched)
    if _tp_rank() != 0:
        return
    sched._connex_ep_q = queue.Queue()
    sched._connex_ep_wait = {}
    _serve(sched, int(os.environ.get("CONNEX_EP_PORT") or 0))
    _advertise(sched)


def ctl_file(server_port) -> str:
    """Where TP rank 0 advertises the control endpoint of the server on
    ``server_port`` (``CONNEX_EP_CTL_FILE`` overrides)."""
    return os.environ.get("CONNEX_EP_CTL_FILE") or os.path.join(tempfile.gettempdir(),
                                                                f"connex-ep-ctl-{server_port}.json")


def _server_port(sched):
    port = getattr(getattr(sched, "server_args", None), "port", None)
    if port is None:
        try:
            from sglang.srt.runtime_context import get_serving
            port = getattr(get_serving(), "port", None)
        except Exception:  # noqa: BLE001
            port = None
    return port


def _advertise(sched) -> dict:
    host, port = sched._connex_ep_srv.server_address[:2]
    info = {"url": f"http://{host}:{port}", "port": port, "server_port": _server_port(sched), "pid": os.getpid()}
    path = ctl_file(info["server_port"])
    with open(path + ".tmp", "w") as f:
        json.dump(info, f)
    os.replace(path + ".tmp", path)
    sched._connex_ep_ctl = info
    log.info("connex.ep control endpoint %s (advertised in %s)", info["url"], path)
    return info


def _run_cmd(sched, cmd: ConnexEPCmd) -> None:
    """Runs on every TP rank at the same point of the scheduler loop; rank 0
    hands the gathered per-rank results to the waiting HTTP request."""
    import torch.distributed as dist
    t0 = time.perf_counter()
    try:
        if not cmd.method.startswith("connex_ep_"):
            raise AttributeError(f"not a connex.ep command: {cmd.method}")
        res = {"ok": True, "result": getattr(sched._connex_ep, cmd.method)(*cmd.args)}
    except Exception as ex:  # noqa: BLE001
        log.exception("connex.ep %s failed", cmd.method)
        res = {"ok": False, "error": repr(ex)}
    res["rank_s"] = time.perf_counter() - t0
    res["queue_s"] = time.time() - cmd.t_enq
    group = getattr(sched, "tp_cpu_group", None)
    n = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
    out = [res]
    if n > 1:
        out = [None] * n
        dist.all_gather_object(out, res, group=group)
    waiting = getattr(sched, "_connex_ep_wait", None)
    slot = waiting.pop(cmd.seq, None) if waiting is not None else None
    if slot is not None:
        slot["res"] = out
        slot["ev"].set()


def _serve(sched, port: int) -> ThreadingHTTPServer:
    counter = [0]
    lock = threading.Lock()

    class Handler(BaseHTTPRequestHandler):
        def log_message(self, *a):
            pass

        def _send(self, code: int, body) -> None:
            data = json.dumps(body).encode()
            self.send_response(code)
            self.send_header("Content-Type", "application/json")
            self.send_header("Content-Length", str(len(data)))
            self.end_headers()
            self.wfile.write(data)

        def do_GET(self):
            self._send(200, {"ok": True})

        def do_POST(self):
            try:
                req = json.loads(self.rfile.read(int(self.headers.get("Content-Length") or 0)) or b"{}")
                method = req["method"]
            except (ValueError, KeyError) as ex:
                return self._send(400, {"error": repr(ex)})
            with lock:
                counter[0] += 1
                seq = counter[0]
            slot = {"ev": threading.Event(), "res": None}
            sched._connex_ep_wait[seq] = slot
            sched._connex_ep_q.put(ConnexEPCmd(seq, method, req.get("args") or []))
            if not slot["ev"].wait(float(req.get("timeout", 120))):
                sched._connex_ep_wait.pop(seq, None)
                return self._send(504, {"error": "timeout"})
            self._send(200, {"results": slot["res"]})

    srv = ThreadingHTTPServer((os.environ.get("CONNEX_EP_HOST", "127.0.0.1"), port), Handler)
    srv.daemon_threads = True
    threading.Thread(target=srv.serve_forever, daemon=True, name="connex-ep-ctl").start()
    sched._connex_ep_srv = srv
    return srv


class SGLangEPWorker(EPWorkerCore):
    """Per-scheduler EP state; the RPCs are :class:`EPWorkerCore`'s."""

    def __init__(self, sched):
        self.sched = sched

    # ---- engine access ------------------------------------------------------
    def _md(self):
        from sglang.srt.eplb.expert_location import get_global_expert_location_metadata
        md = get_global_expert_location_metadata()
        if md is None:
            raise RuntimeError("no expert location metadata: EP is off or the model has no EPLB support")
        return md

    def _ep_rank(self) -> int:
        from sglang.srt.runtime_context import get_parallel
        return get_parallel().moe_ep_rank

    def _dispatch(self) -> str:
        from sglang.srt.runtime_context import get_exec
        return get_exec().moe.ep_dispatch_algorithm

    def _ep_maps(self) -> EngineMaps:
        md = self._md()
        if md.logical_to_all_physical_map.shape[0] == 0:
            raise RuntimeError("empty expert location metadata")
        return EngineMaps(md.physical_to_logical_map, md.logical_to_all_physical_map,
                          md.logical_to_all_physical_map_num_valid, num_ranks=md.ep_size,
                          slots_per_rank=md.num_local_physical_experts, num_experts=md.num_logical_experts,
                          p2l_cpu=md.physical_to_logical_map_cpu, l2p_cpu=md.logical_to_all_physical_map_cpu,
                          rank_pick=md.logical_to_rank_dispatch_physical_map, dispatch=self._dispatch())

    def _ep_order_writes(self, stream) -> None:
        fwd = getattr(getattr(self, "sched", None), "forward_stream", None)
        if fwd is not None and fwd != stream:
            stream.wait_stream(fwd)

    def _expert_layers(self) -> list:
        """Per MoE layer id: the expert parameters viewed as ``[local slots,
        ...]`` (fused shared-expert rows past the routed slots excluded)."""
        cached = self.__dict__.get("_cx_layers")
        if cached is not None:
            return cached
        from sglang.srt.layers.moe.fused_moe_triton.layer import FusedMoE
        md = self._md()
        S = md.num_local_physical_experts
        found = {}
        for mod in self.sched.tp_worker.model_runner.model.modules():
            if isinstance(mod, FusedMoE) and getattr(mod, "layer_id", None) is not None:
                n = mod.num_local_experts
                found[mod.layer_id] = [p.data[:S] for _, p in mod.named_parameters(recurse=False)
                                       if p.dim() >= 1 and p.shape[0] == n]
        missing = [l for l in range(md.num_layers) if l not in found]
        if missing:
            raise RuntimeError(f"layers {missing[:4]} have no FusedMoE (dense layers are not supported)")
        self.__dict__["_cx_layers"] = [found[l] for l in range(md.num_layers)]
        return self.__dict__["_cx_layers"]

    def _ep_load_counts(self):
        """Tokens per physical slot in SGLang's expert distribution recorder
        (``--expert-distribution-recorder-mode stat``; None otherwise)."""
        try:
            from sglang.srt.eplb.expert_distribution import get_global_expert_distribution_recorder
            acc = getattr(get_global_expert_distribution_recorder(), "_accumulator", None)
            data = getattr(acc, "_global_physical_count_of_buffered_step", None)
            return None if data is None else data.get_all().sum(dim=0).sum(dim=0).cpu().tolist()
        except Exception:  # noqa: BLE001
            return None


class SGLangEPEngine(HTTPEPEngine):
    """``EPController`` engine handle for one SGLang server (all EP ranks),
    talking to TP rank 0's control endpoint."""

    path = "/rpc"

    @classmethod
    def from_server(cls, server_url: str, **kw) -> "SGLangEPEngine":
        """Handle for the SGLang server at ``server_url`` on this host (reads
        the endpoint its TP rank 0 advertised)."""
        port = int(server_url.rstrip("/").rsplit(":", 1)[1])
        with open(ctl_file(port)) as f:
            return cls(json.load(f)["url"], **kw)

    def _unwrap(self, method: str, body):
        out = body["results"]
        errs = [x["error"] for x in out if not x["ok"]]
        if errs:
            raise RuntimeError(f"{method} failed: {errs}")
        self.last.setdefault("rank_s", {})[method] = [x["rank_s"] for x in out]
        self.last.setdefault("queue_s", {})[method] = out[0].get("queue_s")
        return [x["result"] for x in out]


__all__ = ["register", "install", "ConnexEPCmd", "SGLangEPWorker", "SGLangEPEngine", "ctl_file"]
