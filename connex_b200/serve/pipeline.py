"""Joining an elastic pipeline from a serving process: the stage endpoint,
its data plane and its directory membership.

Data planes: ``link`` -- elastic NCCL pair links (GPU to GPU over NVLink
inside a box), rendezvous through a ``torch.distributed`` TCP store that
stage 0 replica 0 hosts (``--store HOST:PORT``); ``inline`` -- tensor bytes
inside the ZeroMQ messages (no store, any network, for small or CPU runs).
Membership: the directory / front router (``connex-directory`` or
``connex-front-router``) lists the replicas of every stage; a replica that
dies is deregistered (lease) and stage 0 fails over to another replica of
the next stage, re-prefilling the rows whose KV it does not hold.

Liveness (``watch=True``): every process also runs a native transfer engine
whose URL it lists as ``cx=<url>`` beside its step address; each stage
connects to the engines of the next stage's replicas and fails over on a
peer-death event within milliseconds, before any lease expires.  Stages 1..
answer the liveness protocol (:class:`connex.pp.liveness.StageResponder`:
READY after a restart, DYING on a clean exit); stage 0 runs the step
watchdog (:func:`watchdog`).
"""
from __future__ import annotations

import logging
from datetime import timedelta
from typing import Optional, Tuple

log = logging.getLogger("connex_b200.serve.pipeline")


def split_layers(num_layers: int, num_stages: int, spec: Optional[str] = None) -> list:
    """Layer ranges of the stages: ``spec`` lists the first layer of stages
    1.. (e.g. ``"16"`` for 32 layers over 2 stages); even split otherwise."""
    if spec:
        starts = [0] + [int(x) for x in spec.split(",") if x.strip()]
    else:
        starts = [num_layers * s // num_stages for s in range(num_stages)]
    if len(starts) != num_stages or starts != sorted(set(starts)) or starts[-1] >= num_layers:
        raise ValueError(f"bad stage split {starts} for {num_layers} layers over {num_stages} stages")
    return [(a, b) for a, b in zip(starts, starts[1:] + [num_layers])]


def join(model: str, stage: int, num_stages: int, replica: int, device, directory: str, data: str = "link",
         store: Optional[str] = None, store_master: bool = False, host: str = "127.0.0.1",
         recv_timeout_s: float = 30.0, heartbeat_s: float = 0.5, watch: bool = True,
         state_dir: Optional[str] = None) -> Tuple[object, object]:
    """(endpoint, directory client) of this stage replica, registered."""
    import torch.distributed as dist

    from connex.directory import DirectoryClient
    from connex.pp.endpoint import ENGINE_ADDRESS_PREFIX, PipelineEndpoint
    from connex.pp.membership import DirectoryMembership
    ep = PipelineEndpoint(model, stage, num_stages, replica, data=data, device=str(device), host=host,
                          recv_timeout_s=recv_timeout_s)
    addresses = [ep.address]
    ep.liveness_engine = _liveness_engine(model, stage, replica, host) if watch else None
    if ep.liveness_engine is not None:
        addresses.append(ENGINE_ADDRESS_PREFIX + ep.liveness_engine.local_url)
    if data == "link":
        from connex_b200.parallel.pplink import PairLinks
        if not store:
            raise ValueError("the link data plane needs --store HOST:PORT")
        h, p = store.rsplit(":", 1)
        st = dist.TCPStore(h, int(p), is_master=store_master, wait_for_workers=False, timeout=timedelta(seconds=60))
        ep.links = PairLinks(dist.PrefixStore("pplinks/", st), ep.link_id, device, timeout_s=60)
        ep._store = st                      # kept alive with the endpoint
    client = DirectoryClient(directory, model, stage, replica_idx=replica, local_addresses=addresses)
    client.start()
    client.start_event_listener()
    ep.attach_membership(DirectoryMembership(client, num_stages))
    ep.responder = None
    if stage > 0:
        from connex.pp.liveness import StageResponder
        ep.responder = StageResponder(ep, state_dir=state_dir)
    client.register(addresses)
    client.start_heartbeat(heartbeat_s)
    if ep.liveness_engine is not None and stage + 1 < num_stages:
        ep.watch_peers(ep.liveness_engine)          # the listed replicas of the next stage, and later joiners
    if ep.responder is not None:
        ep.responder.announce()                     # READY to the stage-0 instances served before a restart
    return ep, client


def _liveness_engine(model: str, stage: int, replica: int, host: str):
    """This process's native engine for peer events (None without the extension)."""
    try:
        from connex_b200.engine import Engine
    except ImportError as e:
        log.warning("no native engine (%s): failures are found by leases and step timeouts only", e)
        return None
    return Engine(model, stage, 0, replica, listen_ip=host)


def watchdog(ep, link, client=None, **kw):
    """Stage 0's step watchdog over ``link`` (a :class:`connex.pp.link.Stage0Link`),
    reporting failures further down the chain to the directory; started."""
    from connex.pp.liveness import ChainWatchdog
    report = None
    if client is not None:
        def report(stage, replica, reason):
            client.report_failure((ep.model, stage, 0, replica))
    return ChainWatchdog(ep, link, report=report, **kw).start()


def leave(ep, client, reason: str = "exiting") -> None:
    """Leave the pipeline: DYING to the owner (stages 1..), deregister, close."""
    try:
        if getattr(ep, "watchdog", None) is not None:
            ep.watchdog.stop()
        if getattr(ep, "responder", None) is not None:
            ep.responder.dying(reason)
        client.deregister()
        client.stop()
    finally:
        ep.close()
        if ep.links is not None:
            ep.links.close()
        if getattr(ep, "liveness_engine", None) is not None:
            ep.liveness_engine.close()
