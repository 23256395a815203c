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
"""
from __future__ import annotations

from datetime import timedelta
from typing import Optional, Tuple


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
         recv_timeout_s: float = 30.0, heartbeat_s: float = 0.5) -> Tuple[object, object]:
    """(endpoint, directory client) of this stage replica, registered."""
    import torch.distributed as dist

    from connex.directory import DirectoryClient
    from connex.pp.endpoint import PipelineEndpoint
    from connex.pp.membership import DirectoryMembership
    ep = PipelineEndpoint(model, stage, num_stages, replica, data=data, device=str(device), host=host,
                          recv_timeout_s=recv_timeout_s)
    if data == "link":
        from connex_b200.parallel.pplink import PairLinks
        if not store:
            raise ValueError("the link data plane needs --store HOST:PORT")
        h, p = store.rsplit(":", 1)
        st = dist.TCPStore(h, int(p), is_master=store_master, wait_for_workers=False, timeout=timedelta(seconds=60))
        ep.links = PairLinks(dist.PrefixStore("pplinks/", st), ep.link_id, device, timeout_s=60)
        ep._store = st                      # kept alive with the endpoint
    client = DirectoryClient(directory, model, stage, replica_idx=replica, local_addresses=[ep.address])
    client.start()
    client.start_event_listener()
    ep.attach_membership(DirectoryMembership(client, num_stages))
    client.register([ep.address])
    client.start_heartbeat(heartbeat_s)
    return ep, client


def leave(ep, client) -> None:
    try:
        client.deregister()
        client.stop()
    finally:
        ep.close()
        if ep.links is not None:
            ep.links.close()
