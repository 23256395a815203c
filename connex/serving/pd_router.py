"""PD router: prefill, then decode, over elastic prefill and decode pools.

vLLM mode, per request: the prompt goes to a prefill instance with
``max_tokens=1`` and ``kv_transfer_params={"do_remote_decode": true,
"transfer_id": ...}``; the ``kv_transfer_params`` of its answer then go with
the streamed request to a decode instance, which pulls the prompt's KV.
SGLang mode sends prefill and decode together, paired by a
``bootstrap_room``; the prefill's outcome guards the decode's first token.

Pools (:class:`ElasticPool`) are the union of static URLs, a file re-read
every second and the front router's PD registrations; a new member takes
traffic once a probe succeeded; ``POST /pd/drain`` / ``/pd/undrain``
(loopback or a bearer token) stop / resume new traffic to a member.

Failures, on top of the resume proxy (:mod:`connex.serving.proxy`):

* a failed prefill is retried on another prefill instance;
* a decode that fails before its first token while it still answers probes
  failed its KV hand-off: prefill again elsewhere, without blaming it;
* a decode that dies after k tokens resumes on another decode instance with
  prompt + k ids and ``max_tokens - k``, re-pulling the held KV when its
  prefill instance still holds it, else prefilling the extended prompt;
* a front-router failure event (``connex.endpoint_deregistered`` with a
  failure reason) cuts the member's streams at once.

Behavioural parity: ``connex/serving/pd_router.py:68-559`` of the reference
(routes, flags, request fields); the structure here is this module's own.
"""
from __future__ import annotations

import argparse
import asyncio
import hmac
import json
import logging
import os
import time
import uuid
from typing import Dict, List, Optional, Set, Tuple

import aiohttp
from aiohttp import web

from connex.serving.proxy import RETRYABLE, Endpoint, Pool, Proxy, Resumer, StreamBroken, UpstreamFailed

log = logging.getLogger("connex.pd_router")

UNPROBED = 1e18      # bad_until of a member that has not answered a probe yet
_NOT_FOR_PREFILL = ("stream_options", "logprobs", "top_logprobs", "return_tokens_as_token_ids", "min_tokens",
                    "kv_transfer_params")


class ElasticPool(Pool):
    """Members from three sources -- static URLs, an endpoints file, a dynamic
    list (the front router's registrations) -- minus drained members; a new
    member starts unprobed (no traffic) unless ``probe_new`` is off."""

    def __init__(self, urls=(), endpoints_file=None, blacklist_s: float = 5.0, probe_new: bool = True):
        self.static = [u.strip().rstrip("/") for u in urls if u.strip()]
        self.dynamic: List[str] = []
        self.drained: Set[str] = set()
        self.probe_new = probe_new
        super().__init__(self.static, endpoints_file, blacklist_s)

    def set_urls(self, urls) -> None:
        merged = list(dict.fromkeys(u.strip().rstrip("/") for u in urls if u.strip()))
        for u in merged:
            if u not in self.eps:
                ep = self.eps[u] = Endpoint(u)
                if self.probe_new:
                    ep.bad_until = UNPROBED
        listed = [u for u in merged if u not in self.drained]
        if listed != self.order:
            log.info("pool: +%s -%s", sorted(set(listed) - set(self.order)), sorted(set(self.order) - set(listed)))
        self.order = listed

    def refresh(self) -> None:
        from_file = (self._file_urls() or []) if self.file else []
        self.set_urls(self.static + from_file + self.dynamic)

    def set_dynamic(self, urls) -> None:
        self.dynamic = list(urls)
        self.refresh()

    def reload(self) -> None:
        self.refresh()

    def drain(self, url: str) -> None:
        url = url.rstrip("/")
        self.drained.add(url)
        self.order = [u for u in self.order if u != url]

    def undrain(self, url: str) -> None:
        self.drained.discard(url.rstrip("/"))
        self.refresh()

    def healthy_urls(self) -> List[str]:
        now = time.monotonic()
        return [u for u in self.order if self.eps[u].healthy(now)]


class PrefillFailed(UpstreamFailed):
    pass


class PDResumer(Resumer):
    """A request with its prompt KV: ``kv`` (the ``kv_transfer_params`` the
    decode pulls with), the prefill instance holding it (``kv_ep``) and the
    completion tokens already out when it was made (``kv_tokens``)."""

    def __init__(self, proxy, kind, body):
        super().__init__(proxy, kind, body)
        self.kv: Optional[dict] = None
        self.kv_ep: Optional[Endpoint] = None
        self.kv_tokens = 0
        self.prefills = 0
        self.avoid_prefill: Optional[Endpoint] = None   # the next prefill goes elsewhere
        self.prefill_task: Optional[asyncio.Future] = None  # SGLang: the paired prefill request
        self._guard = None

    def _kv_reusable(self) -> bool:
        """The held prompt KV serves the next decode attempt only while its
        holder lives and the new prompt extends it id for id."""
        if self.kv_ep is None or not self.kv_ep.healthy(time.monotonic()):
            return False
        return self.k == self.kv_tokens or (self.use_ids and not self.chat)

    async def build(self, ep):
        b = await super().build(ep)
        if self.p.engine == "sglang":
            await self.p.sglang_dispatch(self, b)
            return b
        if self.kv is not None:
            if not self._kv_reusable():
                self.kv = None
            elif self.k > 0:
                self.p.stats["kv_repulls"] += 1
        if self.kv is None:
            self.kv, self.kv_ep = await self.p.prefill(self, b)
            self.kv_tokens = self.k
        b["kv_transfer_params"] = dict(self.kv)
        return b

    def first_token_guard(self):
        return self._guard


class PDRouter(Proxy):
    resumer_cls = PDResumer

    def __init__(self, prefill: ElasticPool, decode: ElasticPool, front_router: Optional[str] = None,
                 model: Optional[str] = None, membership_interval: float = 0.5, prefill_timeout=None,
                 engine: str = "vllm", bootstrap: Optional[dict] = None, bootstrap_port: int = 8998,
                 front_router_events: Optional[str] = None, **kw):
        super().__init__(decode, **kw)
        if engine not in ("vllm", "sglang"):
            raise ValueError(f"engine must be vllm or sglang, got {engine!r}")
        self.engine = engine
        self.bootstrap = dict(bootstrap or {})
        self.bootstrap_port = bootstrap_port
        self.prefill_pool = prefill
        self.front_router = front_router
        self.model = model
        self.membership_interval = membership_interval
        self.prefill_timeout = prefill_timeout
        if front_router and not front_router_events:
            front_router_events = front_router.rsplit(":", 1)[0] + ":15560"
        self.front_router_events = front_router_events
        self.admin_token = os.getenv("CONNEX_PD_ADMIN_TOKEN") or None
        self._members: Dict[Tuple[str, int], str] = {}      # (role, replica) -> URL
        self.stats.update({"prefills": 0, "prefill_retries": 0, "kv_reprefills": 0, "kv_repulls": 0,
                           "membership_errors": 0, "failure_events": 0})

    def app(self):
        app = super().app()
        app.router.add_get("/pd/pools", self.handle_pools)
        app.router.add_post("/pd/drain", self.handle_drain)
        app.router.add_post("/pd/undrain", self.handle_undrain)
        return app

    async def _startup(self, app=None):
        await super()._startup(app)
        if self.prefill_pool.file:
            self._background(self._every(1.0, self.prefill_pool.reload))
        if self.front_router:
            self._background(self._membership_loop())
            if self.front_router_events:
                self._background(self._failure_events_loop())

    def _pool_of(self, role_or_ep) -> ElasticPool:
        if isinstance(role_or_ep, Endpoint):
            return self.prefill_pool if role_or_ep.url in self.prefill_pool.eps else self.pool
        return self.prefill_pool if role_or_ep == "prefill" else self.pool

    # ------------------------------------------------------------ membership
    def _apply_membership(self, pools) -> None:
        from connex.protocol import PDRole
        for m in pools[PDRole.PREFILL]:
            if m.kv_addr:
                self.bootstrap[m.url] = m.kv_addr
        for role in (PDRole.PREFILL, PDRole.DECODE):
            for m in pools[role]:
                self._members[(role, m.replica)] = m.url
        self.prefill_pool.set_dynamic([m.url for m in pools[PDRole.PREFILL]])
        self.pool.set_dynamic([m.url for m in pools[PDRole.DECODE]])

    async def _membership_loop(self):
        from connex.pd.membership import fetch_pools
        loop = asyncio.get_running_loop()
        while True:
            pools = await loop.run_in_executor(None, fetch_pools, self.front_router, self.model)
            if pools is None:
                self.stats["membership_errors"] += 1
            else:
                self._apply_membership(pools)
            await asyncio.sleep(self.membership_interval)

    def on_failure_event(self, ev: dict) -> bool:
        """A front-router event; True when it cut a member.  Only
        deregistrations with a failure reason count (a graceful leave lets
        in-flight requests finish)."""
        from connex.pd.membership import STAGE_ROLE
        payload = ev.get("payload") or {}
        reason = payload.get("reason")
        if not reason or reason in ("group_left", "expired"):
            return False
        lid = payload.get("lid") or {}
        role = STAGE_ROLE.get(lid.get("stage_idx"))
        url = self._members.get((role, lid.get("replica_idx")))
        pool = self._pool_of(role)
        ep = pool.eps.get(url) if url is not None else None
        if ep is None or not ep.healthy(time.monotonic()):
            return False
        self.stats["failure_events"] += 1
        pool.mark_bad(ep, f"front-router: {reason}")
        return True

    async def _failure_events_loop(self):
        import zmq
        import zmq.asyncio
        sub = zmq.asyncio.Context.instance().socket(zmq.SUB)
        sub.setsockopt(zmq.LINGER, 0)
        sub.setsockopt(zmq.SUBSCRIBE, b"connex.endpoint_deregistered")
        sub.connect(self.front_router_events)
        try:
            while True:
                try:
                    _, data = await sub.recv_multipart()
                    self.on_failure_event(json.loads(data))
                except (ValueError, zmq.ZMQError):
                    continue
        finally:
            sub.close(0)

    # ---------------------------------------------------------------- probes
    def _probe_targets(self) -> List[tuple]:
        return [(e, p) for p in (self.pool, self.prefill_pool) for e in list(p.eps.values()) if e.url in p.order]

    async def _probe_loop(self):
        while True:         # probe right away: new members wait for their first probe
            await asyncio.gather(*(self._probe(e, p) for e, p in self._probe_targets()), return_exceptions=True)
            await asyncio.sleep(self.probe_interval)

    async def _probe(self, ep: Endpoint, pool: Optional[Pool] = None) -> None:
        pool = pool or self._pool_of(ep)
        if ep.bad_until >= UNPROBED:          # a new member: one answer admits it
            if await self._alive(ep):
                log.info("member %s is up", ep.url)
                pool.mark_good(ep)
            return
        await super()._probe(ep, pool)

    # --------------------------------------------------------------- prefill
    def _prefill_body(self, body: dict) -> dict:
        req = {k: v for k, v in body.items() if k not in _NOT_FOR_PREFILL}
        req["stream"] = False
        req["max_tokens"] = 1
        if "max_completion_tokens" in req:
            req["max_completion_tokens"] = 1
        return req

    async def _post_json(self, url: str, body: dict):
        async with self.session.post(url, json=body, timeout=aiohttp.ClientTimeout(total=self.prefill_timeout)) as r:
            try:
                return r.status, await r.json(content_type=None)
            except ValueError:
                return r.status, None

    async def _prefill_on(self, st: PDResumer, ep: Endpoint, req: dict) -> dict:
        """One prefill attempt; its ``kv_transfer_params`` or StreamBroken.
        A member declared dead meanwhile ends the attempt at once."""
        call = asyncio.ensure_future(self._post_json(ep.url + self._path(st), req))
        watch = {call}
        if ep.healthy(time.monotonic()):
            watch.add(asyncio.ensure_future(ep.dead.wait()))
        try:
            done, _ = await asyncio.wait(watch, return_when=asyncio.FIRST_COMPLETED)
        finally:
            for t in watch - {call}:
                t.cancel()
        if call not in done:
            call.cancel()
            raise StreamBroken("prefill instance died")
        status, data = call.result()
        if status != 200:
            raise StreamBroken(f"prefill HTTP {status}: {str(data)[:200]}")
        kv = (data or {}).get("kv_transfer_params")
        if not kv:
            raise StreamBroken("prefill response without kv_transfer_params (not a KV producer?)")
        if st.prompt_tokens is None:
            st.prompt_tokens = (data.get("usage") or {}).get("prompt_tokens")
        return kv

    async def prefill(self, st: PDResumer, body: dict):
        """Prefill ``body`` somewhere; returns (kv_transfer_params, endpoint)."""
        req = self._prefill_body(body)
        tried = [st.avoid_prefill.url] if st.avoid_prefill is not None else []
        st.avoid_prefill = None
        pool, last = self.prefill_pool, "no prefill instances"
        for n in range(max(self.max_attempts, len(pool.order) + 1)):
            ep = pool.pick(exclude=tried) or pool.pick()
            if ep is None:
                break
            self.stats["prefill_retries"] += n > 0
            req["kv_transfer_params"] = {"do_remote_decode": True, "do_remote_prefill": False,
                                         "transfer_id": uuid.uuid4().hex}
            ep.inflight += 1
            st.prefills += 1
            try:
                kv = await self._prefill_on(st, ep, req)
                self.stats["prefills"] += 1
                pool.mark_good(ep)      # it just answered: a blacklisted last resort is back
                return kv, ep
            except (StreamBroken, ValueError, *RETRYABLE) as e:
                last = f"{type(e).__name__}: {e}"
                pool.mark_bad(ep, last)
                tried.append(ep.url)
                log.warning("prefill on %s failed: %s", ep.url, last)
            finally:
                ep.inflight -= 1
        raise PrefillFailed(f"prefill failed: {last}", st)

    # ---------------------------------------------------------------- SGLang
    def _bootstrap_of(self, url: str):
        addr = self.bootstrap.get(url)
        if addr:
            host, port = addr.rsplit(":", 1)
            return host, int(port)
        from urllib.parse import urlparse
        return urlparse(url).hostname, self.bootstrap_port

    async def _sglang_prefill(self, pep: Endpoint, path: str, body: dict) -> Optional[str]:
        """The paired prefill request; None when it succeeded, else why not."""
        pep.inflight += 1
        try:
            async with self.session.post(pep.url + path, json=body,
                                         timeout=aiohttp.ClientTimeout(total=self.prefill_timeout)) as r:
                await r.read()
                return None if r.status == 200 else f"prefill HTTP {r.status}"
        except RETRYABLE as e:
            self.prefill_pool.mark_bad(pep, f"{type(e).__name__}: {e}")
            return f"prefill {type(e).__name__}"
        finally:
            pep.inflight -= 1

    async def sglang_dispatch(self, st: PDResumer, b: dict) -> None:
        """Pick a prefill, pair it with this decode attempt by a bootstrap
        room, start the prefill and guard the decode's first token with it."""
        avoid = [st.avoid_prefill.url] if st.avoid_prefill is not None else []
        st.avoid_prefill = None
        pep = self.prefill_pool.pick(exclude=avoid) or self.prefill_pool.pick()
        if pep is None:
            raise PrefillFailed("no prefill instances", st)
        host, port = self._bootstrap_of(pep.url)
        b.update(bootstrap_host=host, bootstrap_port=port, bootstrap_room=uuid.uuid4().int & ((1 << 63) - 1))
        prefill_body = {k: v for k, v in b.items() if k != "stream_options"}
        prefill_body["stream"] = False
        st.kv_ep = pep
        st.prefills += 1
        self.stats["prefills"] += 1
        st.prefill_task = asyncio.ensure_future(self._sglang_prefill(pep, self._path(st), prefill_body))
        task = st.prefill_task

        async def guard():
            why = await asyncio.shield(task)
            if why is None:
                await asyncio.Event().wait()     # the prefill succeeded: never abort the decode
            return why
        st._guard = guard

    # ---------------------------------------------------------------- decode
    async def on_attempt_failed(self, st: PDResumer, ep: Endpoint, err: BaseException, produced: int) -> bool:
        if self.engine == "sglang":
            pt = st.prefill_task
            if pt is not None and pt.done() and not pt.cancelled() and pt.result():
                st.avoid_prefill = st.kv_ep           # the paired prefill failed, not the decode
                self.stats["prefill_retries"] += 1
                if produced == 0:
                    return False
            elif produced > 0:
                self.stats["kv_reprefills"] += 1
        elif produced == 0 and st.kv is not None and await self._alive(ep):
            # the decode answers and produced nothing: its KV hand-off failed; prefill again
            st.avoid_prefill = st.kv_ep
            st.kv = None
            self.stats["kv_reprefills"] += 1
            log.warning("decode %s failed before its first token; re-prefilling", ep.url)
            return False
        return await super().on_attempt_failed(st, ep, err, produced)

    # ----------------------------------------------------------------- admin
    async def handle_pools(self, request):
        now = time.monotonic()

        def describe(p: ElasticPool):
            listed = [{"url": u, "healthy": p.eps[u].healthy(now), "probed": p.eps[u].bad_until < UNPROBED,
                       "inflight": p.eps[u].inflight} for u in p.order]
            return listed + [{"url": u, "drained": True, "inflight": p.eps[u].inflight}
                             for u in p.drained if u in p.eps]
        return web.json_response({"prefill": describe(self.prefill_pool), "decode": describe(self.pool)})

    def _admin_allowed(self, request) -> bool:
        """Pool changes: loopback clients, or ``Authorization: Bearer <token>``
        when an admin token is configured."""
        if self.admin_token:
            got = request.headers.get("Authorization", "")
            if hmac.compare_digest(got.encode(), f"Bearer {self.admin_token}".encode()):
                return True
        remote = (request.remote or "").split("%", 1)[0]
        return remote in ("127.0.0.1", "::1", "localhost") or remote.startswith("::ffff:127.")

    async def _admin(self, request, action: str):
        if not self._admin_allowed(request):
            raise web.HTTPForbidden(text="pool admin needs loopback or an admin token")
        body = await request.json()
        url, role = body.get("url", ""), body.get("role")
        for name, p in (("prefill", self.prefill_pool), ("decode", self.pool)):
            if role in (None, name):
                getattr(p, action)(url)
        return web.json_response({"ok": True})

    async def handle_drain(self, request):
        return await self._admin(request, "drain")

    async def handle_undrain(self, request):
        return await self._admin(request, "undrain")


def main() -> None:
    ap = argparse.ArgumentParser(description="PD router over elastic prefill / decode pools")
    ap.add_argument("--host", default="0.0.0.0")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--prefill", default="")
    ap.add_argument("--decode", default="")
    ap.add_argument("--prefill-file", default=None)
    ap.add_argument("--decode-file", default=None)
    ap.add_argument("--front-router", default=None, help="tcp://host:port of the front-router API")
    ap.add_argument("--model", default=None)
    ap.add_argument("--front-router-events", default=None)
    ap.add_argument("--engine", choices=["vllm", "sglang"], default="vllm")
    ap.add_argument("--bootstrap", default="", help="SGLang: prefill_url=host:port,...")
    ap.add_argument("--bootstrap-port", type=int, default=8998)
    ap.add_argument("--membership-interval", type=float, default=0.5)
    ap.add_argument("--idle-timeout", type=float, default=5.0)
    ap.add_argument("--first-token-timeout", type=float, default=None)
    ap.add_argument("--prefill-timeout", type=float, default=None)
    ap.add_argument("--connect-timeout", type=float, default=2.0)
    ap.add_argument("--max-attempts", type=int, default=4)
    ap.add_argument("--blacklist-s", type=float, default=5.0)
    ap.add_argument("--probe-interval", type=float, default=0.5)
    ap.add_argument("--admin-token", default=None)
    ap.add_argument("--log-level", default="INFO")
    a = ap.parse_args()
    if a.front_router and not a.model:
        ap.error("--front-router needs --model")
    logging.basicConfig(level=a.log_level, format="%(asctime)s %(name)s %(levelname)s %(message)s")
    router = PDRouter(ElasticPool([u for u in a.prefill.split(",") if u], a.prefill_file, a.blacklist_s),
                      ElasticPool([u for u in a.decode.split(",") if u], a.decode_file, a.blacklist_s),
                      front_router=a.front_router, model=a.model, membership_interval=a.membership_interval,
                      prefill_timeout=a.prefill_timeout, engine=a.engine, bootstrap_port=a.bootstrap_port,
                      front_router_events=a.front_router_events,
                      bootstrap=dict(x.rsplit("=", 1) for x in a.bootstrap.split(",") if x),
                      idle_timeout=a.idle_timeout, connect_timeout=a.connect_timeout, max_attempts=a.max_attempts,
                      probe_interval=a.probe_interval, first_token_timeout=a.first_token_timeout)
    if a.admin_token:
        router.admin_token = a.admin_token
    web.run_app(router.app(), host=a.host, port=a.port, access_log=None)


if __name__ == "__main__":
    main()
