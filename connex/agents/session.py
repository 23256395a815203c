"""Session-aware routing and live session migration for agent workloads.

A session (``session_id`` in the body, or the ``X-Connex-Session`` header)
is a mobile endpoint: logical id ``session/<sid>``, a placement (the
replica holding its prefix state) and an epoch that every move bumps.
Requests of a session stick to its placement.

:meth:`SessionProxy.migrate` moves a session in three steps: a
:class:`KVMover` makes the target hold the session's prefix (the built-in
:class:`ReprefillMover` re-prefills the conversation there so the target's
prefix cache has it), then the epoch is bumped and the placement repointed,
then the session's in-flight generations are cut over with the resume
proxy's :meth:`connex.serving.proxy.Proxy.move`.  A placement that dies is
replaced on the next attempt (failover).  Sessions idle past the TTL are
forgotten.

Behavioural parity: ``connex/agents/session.py:15-264`` of the reference
(routes, header, session fields); the structure here is this module's own.
"""
from __future__ import annotations

import argparse
import logging
import time
from typing import Dict, List, Optional

from aiohttp import web

from connex.serving.proxy import Pool, Proxy, Resumer

log = logging.getLogger("connex.agents")

HEADER = "X-Connex-Session"
_SESSION_FIELD = "_connex_session"          # carries the id from the handler to begin()


class Session:
    __slots__ = ("sid", "url", "epoch", "inflight", "context", "kind", "model", "last_used", "moves")

    def __init__(self, sid: str):
        self.sid = sid
        self.url: Optional[str] = None
        self.epoch = 0
        self.inflight: set = set()
        self.context: Optional[dict] = None     # the last full turn (request + reply) for re-prefill
        self.kind = None
        self.model = None
        self.last_used = time.monotonic()
        self.moves: List[dict] = []

    @property
    def lid(self) -> str:
        return f"session/{self.sid}"

    def info(self) -> dict:
        return {"lid": self.lid, "placement": self.url, "epoch": self.epoch, "inflight": len(self.inflight),
                "moves": self.moves[-5:]}

    def repoint(self, url: str, mode: str, **extra) -> dict:
        """New placement under a new epoch; returns the move record."""
        self.epoch += 1
        rec = {"epoch": self.epoch, "from": self.url, "to": url, "mode": mode, **extra}
        self.url = url
        self.moves.append(rec)
        return rec


def turn_context(st: Resumer) -> dict:
    """The request of a finished turn extended by its reply: what a replica
    must prefill to hold the session's prefix."""
    reply = "".join(st.text)
    b = {k: v for k, v in st.body.items() if k not in ("stream", "stream_options")}
    if st.chat:
        b["messages"] = list(b["messages"]) + [{"role": "assistant", "content": reply}]
        b["add_generation_prompt"] = False
        b["continue_final_message"] = False
    elif st.use_ids and st.prompt_ids is not None and len(st.ids) == st.k:
        b["prompt"] = list(st.prompt_ids) + list(st.ids)
    elif isinstance(b.get("prompt"), str):
        b["prompt"] += reply
    return b


class KVMover:
    """Makes ``dst`` hold ``session``'s prefix state; returns ``{"mode": ...}``
    or raises (the proxy then tries the next mover)."""

    name = "kv"

    async def move(self, proxy, session: Session, src, dst) -> dict:
        raise NotImplementedError


class ReprefillMover(KVMover):
    """Prefill the conversation on ``dst`` (one generated token) so its
    automatic prefix cache holds it before traffic moves."""

    name = "reprefill"
    _DROP = ("stream_options", "logprobs", "return_tokens_as_token_ids", "min_tokens", "max_completion_tokens")

    async def _context(self, proxy, session: Session, dst) -> Optional[dict]:
        resumable = [st for st in session.inflight if st.k > 0 and st.can_resume()]
        if resumable:                      # mid-generation: the prompt plus what was produced so far
            return await resumable[-1].build(proxy.pool.eps[dst])
        return session.context

    async def move(self, proxy, session, src, dst):
        ctx = await self._context(proxy, session, dst)
        if ctx is None:
            return {"mode": self.name, "tokens": 0}
        body = {k: v for k, v in ctx.items() if k not in self._DROP}
        body.update(stream=False, max_tokens=1, temperature=0.0)
        path = "/v1/chat/completions" if session.kind == "chat" else "/v1/completions"
        async with proxy.session.post(dst.rstrip("/") + path, json=body) as r:
            if r.status != 200:
                raise RuntimeError(f"re-prefill on {dst}: HTTP {r.status}")
            out = await r.json()
        return {"mode": self.name, "tokens": (out.get("usage") or {}).get("prompt_tokens")}


class SessionProxy(Proxy):
    def __init__(self, pool: Pool, movers=None, session_ttl_s: float = 3600.0, **kw):
        super().__init__(pool, **kw)
        self.sessions: Dict[str, Session] = {}
        self.movers = list(movers) if movers else [ReprefillMover()]
        self.ttl = session_ttl_s
        self._next_sweep = time.monotonic() + (session_ttl_s or 0)
        self.stats.update(sessions=0, migrations=0, failovers=0)

    def app(self):
        app = super().app()
        app.router.add_get("/sessions", self.handle_sessions)
        app.router.add_post("/sessions/{sid}/migrate", self.handle_migrate)
        app.router.add_post("/sessions/drain", self.handle_drain)
        return app

    async def _handle(self, request, kind):
        body = await request.json()
        sid = body.pop("session_id", None) or request.headers.get(HEADER)
        if sid is not None:
            body[_SESSION_FIELD] = str(sid)
        return await self.respond(request, kind, body)

    # -------------------------------------------------------------- sessions
    def get_session(self, sid: str) -> Session:
        s = self.sessions.get(sid)
        if s is None:
            self.expire_sessions()
            s = self.sessions[sid] = Session(sid)
            self.stats["sessions"] += 1
        return s

    def expire_sessions(self, now: Optional[float] = None) -> int:
        """Forget sessions idle past the TTL (swept at most every TTL/10)."""
        now = time.monotonic() if now is None else now
        if not self.ttl or now < self._next_sweep:
            return 0
        self._next_sweep = now + self.ttl / 10
        idle = [sid for sid, s in self.sessions.items() if not s.inflight and now - s.last_used > self.ttl]
        for sid in idle:
            del self.sessions[sid]
        return len(idle)

    def _session_of(self, st) -> Optional[Session]:
        sid = getattr(st, "sid", None)
        return self.sessions.get(sid) if sid is not None else None

    def begin(self, st):
        st.sid = st.body.pop(_SESSION_FIELD, None)
        if st.sid is None:
            return
        s = self.get_session(st.sid)
        s.inflight.add(st)
        s.kind, s.model, s.last_used = st.kind, st.model, time.monotonic()

    def end(self, st):
        s = self._session_of(st)
        if s is None:
            return
        s.inflight.discard(st)
        s.last_used = time.monotonic()
        if st.finish is not None:
            s.context = turn_context(st)

    def pick(self, st, tried):
        if getattr(st, "sid", None) is None:
            return super().pick(st, tried)
        s = self.get_session(st.sid)
        home = self.pool.eps.get(s.url) if s.url else None
        usable = home is not None and home.url not in tried and home.url in self.pool.order \
            and home.healthy(time.monotonic())
        if usable:
            return home
        ep = self.pool.pick(exclude=tried) or self.pool.pick()
        if ep is None:
            return None
        if s.url is None:
            s.url = ep.url                        # first placement
        elif s.url != ep.url:                     # placement lost: fail over (the new replica re-prefills)
            self.stats["failovers"] += 1
            old = s.url
            s.repoint(ep.url, "failover")
            log.warning("session %s: %s unavailable, failing over to %s (epoch %d)", st.sid, old, ep.url, s.epoch)
        return ep

    # ------------------------------------------------------------- migration
    async def _prepare(self, s: Session, src, target: str, mode: str) -> dict:
        if src == target or mode == "none":
            return {"mode": "none"}
        movers = self.movers if mode == "auto" else [m for m in self.movers if m.name == mode]
        if not movers:
            raise ValueError(f"no mover {mode!r}")
        info = {"mode": "none"}
        for m in movers:
            try:
                return await m.move(self, s, src, target)
            except Exception as e:  # noqa: BLE001 - the next mover
                log.warning("session %s: mover %s failed: %s", s.sid, m.name, e)
                info = {"mode": "none", "error": repr(e)}
        return info

    async def migrate(self, sid: str, target: str, mode: str = "auto") -> dict:
        """Move ``sid`` to ``target``.  ``mode``: "auto" (movers in order), a
        mover name, or "none" (cut over only)."""
        s = self.sessions.get(sid)
        if s is None:
            raise KeyError(sid)
        target = target.rstrip("/")
        if target not in self.pool.eps:
            raise ValueError(f"unknown endpoint {target}")
        src = s.url
        t0 = time.perf_counter()
        info = await self._prepare(s, src, target, mode)
        prepare_s = time.perf_counter() - t0
        rec = s.repoint(target, info.pop("mode"), prepare_s=prepare_s, **info)
        # cut the session's generations over; they resume at the new placement
        rec["inflight_moved"] = sum(self.move(st) for st in list(s.inflight)) if src != target else 0
        self.stats["migrations"] += 1
        return rec

    async def drain(self, url: str, mode: str = "auto") -> List[dict]:
        """Move every session placed on ``url`` elsewhere."""
        url = url.rstrip("/")
        records = []
        for s in [s for s in self.sessions.values() if s.url == url]:
            ep = self.pool.pick(exclude=[url])
            if ep is None or ep.url == url:
                raise RuntimeError("no other endpoint to drain to")
            records.append(await self.migrate(s.sid, ep.url, mode))
        return records

    # --------------------------------------------------------------- routes
    async def handle_sessions(self, request):
        return web.json_response({sid: s.info() for sid, s in self.sessions.items()})

    async def handle_migrate(self, request):
        b = await request.json()
        try:
            rec = await self.migrate(request.match_info["sid"], b["target"], b.get("mode", "auto"))
        except (KeyError, ValueError) as e:
            return web.json_response({"error": str(e)}, status=400)
        return web.json_response(rec)

    async def handle_drain(self, request):
        b = await request.json()
        return web.json_response(await self.drain(b["url"], mode=b.get("mode", "auto")))


def main() -> None:
    ap = argparse.ArgumentParser(description="Session-aware resume proxy")
    ap.add_argument("--host", default="0.0.0.0")
    ap.add_argument("--port", type=int, default=5299)
    ap.add_argument("--endpoints", default="")
    ap.add_argument("--endpoints-file", default=None)
    ap.add_argument("--idle-timeout", type=float, default=30.0)
    ap.add_argument("--probe-interval", type=float, default=1.0)
    ap.add_argument("--no-token-ids", action="store_true")
    ap.add_argument("--log-level", default="INFO")
    a = ap.parse_args()
    logging.basicConfig(level=a.log_level, format="%(asctime)s %(name)s %(levelname)s %(message)s")
    proxy = SessionProxy(Pool([u for u in a.endpoints.split(",") if u], a.endpoints_file),
                         idle_timeout=a.idle_timeout, probe_interval=a.probe_interval, token_ids=not a.no_token_ids)
    web.run_app(proxy.app(), host=a.host, port=a.port, access_log=None)


if __name__ == "__main__":
    main()
