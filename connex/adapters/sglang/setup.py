"""Build a :class:`ConnexPPGroup` for an SGLang stage process from the
environment (reference ``connex/adapters/sglang/setup.py``)::

    PIPELINE_STAGE_IDX, PIPELINE_NUM_STAGES, PIPELINE_REPLICA_IDX
    CONNEX_PP_MODEL (default "default"), CONNEX_ROUTER_PORT (default 5550 + stage)
    FRONT_ROUTER_API / FRONT_ROUTER_EVENTS (the front router this stage registers with)
    CONNEX_PP_INFLIGHT (steps in flight)

Engine-side wiring (not done here)::

    from connex.adapters.sglang import make_pp_group
    scheduler.pp_group = make_pp_group(hooks=MySGLangHooks(scheduler), row_info=scheduler.cx_rows)
"""
from __future__ import annotations

import os
from typing import Any, Callable, Optional

from connex.adapters.sglang.pp_group import ConnexPPGroup


def make_pp_group(hooks: Any = None, row_info: Optional[Callable[[], tuple]] = None, *,
                  stage_idx: Optional[int] = None, num_stages: Optional[int] = None, membership=None,
                  device: str = "cuda", host: str = "127.0.0.1", **endpoint_kw) -> ConnexPPGroup:
    """The endpoint binds ``CONNEX_ROUTER_PORT``; without ``membership`` it
    registers its address with the front router and routes by its table."""
    from connex.pp.endpoint import PipelineEndpoint
    stage = int(os.getenv("PIPELINE_STAGE_IDX", "0")) if stage_idx is None else stage_idx
    n = int(os.getenv("PIPELINE_NUM_STAGES", "1")) if num_stages is None else num_stages
    replica = int(os.getenv("PIPELINE_REPLICA_IDX", "0"))
    model = os.getenv("CONNEX_PP_MODEL", "default")
    port = int(os.getenv("CONNEX_ROUTER_PORT", str(5550 + stage)))
    ep = PipelineEndpoint(model, stage, n, replica, membership=membership, host=host, port=port, device=device,
                          **endpoint_kw)
    if membership is None:
        from connex.epc_client import create_epc_client
        api = os.getenv("FRONT_ROUTER_API", "tcp://127.0.0.1:15555")
        events = os.getenv("FRONT_ROUTER_EVENTS", api.rsplit(":", 1)[0] + ":15560")
        client = create_epc_client(model, stage, front_router_api=api, front_router_events=events,
                                   local_addresses=[ep.address], replica_idx=replica)
        client.start()
        ep.attach_membership(client)
    return ConnexPPGroup(ep, hooks, row_info=row_info)
