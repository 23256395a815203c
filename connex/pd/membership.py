"""PD pool membership through the front router.

Every prefill / decode instance registers ``LID(model, stage=PD_STAGE[role],
shard, replica)`` whose addresses carry its serving URL (``http://...``),
its KV control address (``kv=host:port``) and optionally its transfer-engine
endpoint (``rs=host:port``).  A TP instance is one group of ``group_size``
shards; ``fetch_pools`` lists an instance only while all its shards are
registered.  PD roles map to reserved stage indices (``PD_STAGE``).
Reference: ``connex/pd/membership.py``.
"""
from __future__ import annotations

import logging
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import zmq

from connex.protocol import LogicalEndpointID, PDRole

log = logging.getLogger("connex.pd")

PD_STAGE = {PDRole.PREFILL: 1000, PDRole.DECODE: 1001}
STAGE_ROLE = {v: k for k, v in PD_STAGE.items()}
ROUTE_ACTIVE = 1


def pd_lid(model: str, role: str, replica: int, shard: int = 0) -> LogicalEndpointID:
    return LogicalEndpointID(model, PD_STAGE[role], shard, replica, pd_role=role)


@dataclass
class PDMemberInfo:
    role: str
    replica: int
    url: str
    kv_addr: Optional[str] = None
    extra: List[str] = field(default_factory=list)
    group_size: int = 1


def _gsize(route: dict) -> int:
    return int(route.get("group_size") or (route.get("metadata") or {}).get("group_size") or 1)


def complete_groups(routes: List[dict]) -> List[dict]:
    """Ungrouped routes plus shard 0 of every group whose shards are all active."""
    out, groups = [], {}
    for r in routes:
        lid = r.get("lid") or {}
        if _gsize(r) <= 1:
            out.append(r)
        elif r.get("state", ROUTE_ACTIVE) == ROUTE_ACTIVE:
            groups.setdefault((lid.get("model_name"), lid.get("stage_idx"), lid.get("replica_idx")), {})[
                int(lid.get("shard_idx", 0))] = r
    for shards in groups.values():
        lead = shards.get(0)
        if lead is not None and set(shards) >= set(range(_gsize(lead))):
            out.append(lead)
    return out


def parse_member(route: dict) -> Optional[PDMemberInfo]:
    lid = route.get("lid") or {}
    role = STAGE_ROLE.get(lid.get("stage_idx"))
    if role is None or route.get("state", ROUTE_ACTIVE) != ROUTE_ACTIVE:
        return None
    url, kv, extra = None, None, []
    for a in route.get("addresses") or []:
        if a.startswith(("http://", "https://")):
            url = url or a.rstrip("/")
        elif a.startswith("kv="):
            kv = a[3:]
        else:
            extra.append(a)
    if url is None:
        return None
    return PDMemberInfo(role, int(lid.get("replica_idx", 0)), url, kv, extra, _gsize(route))


def _router_call(front_router_api: str, method: str, params: dict, timeout_ms: int) -> Optional[dict]:
    s = zmq.Context.instance().socket(zmq.REQ)
    s.setsockopt(zmq.LINGER, 0)
    s.setsockopt(zmq.RCVTIMEO, timeout_ms)
    s.setsockopt(zmq.SNDTIMEO, timeout_ms)
    try:
        s.connect(front_router_api)
        s.send_json({"method": method, "params": params})
        return s.recv_json()
    except zmq.ZMQError:
        return None
    finally:
        s.close(0)


def fetch_pools(front_router_api: str, model: str, timeout_ms: int = 2000) -> Optional[Dict[str, List[PDMemberInfo]]]:
    rep = _router_call(front_router_api, "get_routes",
                       {"model_name": model, "stage_idx": list(PD_STAGE.values()), "compact": True}, timeout_ms)
    if rep is None:
        return None
    if "error" in rep:
        log.warning("front router: %s", rep["error"])
        return None
    pools: Dict[str, List[PDMemberInfo]] = {PDRole.PREFILL: [], PDRole.DECODE: []}
    for r in complete_groups(rep.get("routes", [])):
        m = parse_member(r)
        if m is not None:
            pools[m.role].append(m)
    for v in pools.values():
        v.sort(key=lambda m: m.replica)
    return pools


def report_failure(front_router_api: str, lid: LogicalEndpointID, reason: str,
                   timeout_ms: int = 1000) -> Optional[List[str]]:
    """Tell the router that ``lid`` died; it fails the LID's whole group."""
    rep = _router_call(front_router_api, "report_failure",
                       {"lid": {"model_name": lid.model_name, "stage_idx": lid.stage_idx,
                                "shard_idx": lid.shard_idx, "replica_idx": lid.replica_idx},
                        "reason": reason}, timeout_ms)
    return None if rep is None else list(rep.get("failed") or [])


class PDMember:
    """Registers one PD instance (or one TP rank of it) and keeps its lease;
    ``stop()`` deregisters (graceful scale-down)."""

    def __init__(self, front_router_api: str, model: str, role: str, replica: int, http_url: str,
                 kv_addr: Optional[str] = None, heartbeat_interval_s: float = 1.0, events: Optional[str] = None,
                 shard: int = 0, group_size: int = 1, extra_addresses=()):
        from connex.epc_client import EPCV2Client, EPCV2ClientConfig
        addrs = [http_url.rstrip("/")] + ([f"kv={kv_addr}"] if kv_addr else []) + list(extra_addresses)
        cfg = EPCV2ClientConfig(front_router_api=front_router_api,
                                front_router_events=events or front_router_api.rsplit(":", 1)[0] + ":15560",
                                model_name=model, stage_idx=PD_STAGE[role], replica_idx=replica, shard_idx=shard,
                                group_size=group_size, local_addresses=addrs,
                                heartbeat_interval_s=heartbeat_interval_s, ucx_enabled=False)
        self.lid = pd_lid(model, role, replica, shard)
        self.client = EPCV2Client(cfg)

    def start(self) -> bool:
        ok = self.client.start()
        (log.info if ok else log.warning)("PD member %s %s", self.lid, "registered" if ok else "not registered")
        return ok

    def stop(self) -> None:
        self.client.stop()


def _healthy(url: str, timeout_s: float = 2.0) -> bool:
    import urllib.request
    try:
        with urllib.request.urlopen(url.rstrip("/") + "/health", timeout=timeout_s) as r:
            return r.status == 200
    except Exception:  # noqa: BLE001 - not up yet
        return False


def run_member(front_router: str, model: str, role: str, replica: int, url: str, kv_addr: Optional[str] = None,
               shard: int = 0, group_size: int = 1, poll_s: float = 2.0, stop=None, healthy=_healthy) -> int:
    """Sidecar loop for an engine that does not register itself: register
    once ``url``/health answers 200, deregister when it stops answering (the
    engine died or is restarting) and register again when it is back.
    ``stop`` (a ``threading.Event``) ends the loop with a deregistration."""
    import threading
    stop = stop or threading.Event()
    member = None
    while not stop.is_set():
        up = healthy(url)
        if up and member is None:
            member = PDMember(front_router, model, role, replica, url, kv_addr=kv_addr, shard=shard,
                              group_size=group_size)
            if not member.start():
                member.stop()
                member = None
        elif not up and member is not None:
            log.warning("PD member %s: %s/health stopped answering; deregistering", pd_lid(model, role, replica,
                                                                                          shard), url)
            member.stop()
            member = None
        stop.wait(poll_s)
    if member is not None:
        member.stop()
    return 0


def main(argv=None) -> int:
    """``python -m connex.pd.membership --front-router tcp://fr:15555 --model M --role prefill
    --replica 0 --url http://me:8100`` — keeps an engine's PD pool membership
    while its HTTP server is healthy (a sidecar next to a vLLM server with
    the ConnexConnector)."""
    import argparse
    import signal
    import threading
    ap = argparse.ArgumentParser(description="register a PD instance in the front-router pools while it is healthy")
    ap.add_argument("--front-router", required=True)
    ap.add_argument("--model", required=True)
    ap.add_argument("--role", choices=[PDRole.PREFILL, PDRole.DECODE], required=True)
    ap.add_argument("--replica", type=int, default=0)
    ap.add_argument("--url", required=True)
    ap.add_argument("--kv-addr", default=None)
    ap.add_argument("--shard", type=int, default=0)
    ap.add_argument("--group-size", type=int, default=1)
    ap.add_argument("--poll-s", type=float, default=2.0)
    a = ap.parse_args(argv)
    logging.basicConfig(level=logging.INFO, format="%(asctime)s [%(levelname)s] %(name)s: %(message)s")
    stop = threading.Event()
    signal.signal(signal.SIGTERM, lambda *_: stop.set())
    signal.signal(signal.SIGINT, lambda *_: stop.set())
    return run_member(a.front_router, a.model, a.role, a.replica, a.url, a.kv_addr, a.shard, a.group_size,
                      a.poll_s, stop)


if __name__ == "__main__":
    raise SystemExit(main())
