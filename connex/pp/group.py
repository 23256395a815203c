"""Tensor-parallel groups of a pipeline stage (reference ``connex/pp/group.py``).

A TP group is *one* endpoint: its rank 0 registers the stage's LID with
``group_size = tp`` and carries all stage-to-stage traffic; every other rank
registers ``LID(stage, shard=rank)`` with the same ``group_size`` for
liveness only.  The front router fails the whole group when any shard
fails, leaves or stops heartbeating, and the group serves again once all
shards re-registered under the same identity.  The all-reduce inside the
group stays on NCCL over NVLink.
"""
from __future__ import annotations

import logging
import os
from typing import Optional

log = logging.getLogger("connex.pp")


def _router_addrs(front_router_api: Optional[str], events: Optional[str]):
    api = os.getenv("FRONT_ROUTER_API") or os.getenv("CONNEXTE_FRONT_ROUTER_API") or front_router_api \
        or "127.0.0.1:15555"
    if not api.startswith("tcp://"):
        api = "tcp://" + api
    if events is None:
        events = os.getenv("FRONT_ROUTER_EVENTS") or os.getenv("CONNEXTE_FRONT_ROUTER_EVENTS") \
            or api.rsplit(":", 1)[0] + ":15560"
    return api, events


class TPShardMember:
    """Liveness registration of one non-zero TP rank of a pipeline stage."""

    def __init__(self, stage_idx: int, rank: int, tp_size: int, replica_idx: Optional[int] = None,
                 model: Optional[str] = None, front_router_api: Optional[str] = None,
                 events: Optional[str] = None, heartbeat_interval_s: Optional[float] = None):
        from connex.epc_client import EPCV2Client, EPCV2ClientConfig
        if replica_idx is None:
            replica_idx = int(os.getenv("PIPELINE_REPLICA_IDX", "0") or 0)
        model = model or os.getenv("SERVED_MODEL_NAME", "default")
        api, events = _router_addrs(front_router_api, events)
        kw = {} if heartbeat_interval_s is None else {"heartbeat_interval_s": heartbeat_interval_s}
        self.cfg = EPCV2ClientConfig(front_router_api=api, front_router_events=events, model_name=model,
                                     stage_idx=stage_idx, shard_idx=rank, replica_idx=replica_idx,
                                     group_size=tp_size,
                                     local_addresses=[f"tp-shard:{rank}/{tp_size}@{os.getpid()}"],
                                     ucx_enabled=False, **kw)
        self.client = EPCV2Client(self.cfg)

    def start(self) -> bool:
        ok = self.client.start()
        log.info("TP shard %d/%d of stage %d replica %d %s", self.cfg.shard_idx, self.cfg.group_size,
                 self.cfg.stage_idx, self.cfg.replica_idx, "registered" if ok else "failed to register")
        return ok

    def stop(self) -> None:
        self.client.stop()
