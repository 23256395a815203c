"""Port layout of one-stage-per-instance deployments (reference
``connex/adapters/vllm/pp/ports.py``): every downstream stage replica listens
on a control port and one data port per TP rank, and no two (stage, replica,
TP rank) may share a port on a host network::

    control(stage, replica)       = BASE + 1000 * stage + 16 * replica
    data(stage, replica, tp_rank) = control(stage, replica) + 1 + tp_rank

``replica < 62`` and ``tp_rank < 15``; ``BASE`` is ``CONNEX_PP_PORT_BASE``
(47000).  CLI: ``python -m connex.adapters.vllm.pp.ports control|data STAGE
REPLICA [TP_RANK]``.
"""
from __future__ import annotations

import os
import sys
from typing import List, Optional

STAGE_STRIDE = 1000
REPLICA_STRIDE = 16
MAX_REPLICAS = STAGE_STRIDE // REPLICA_STRIDE       # 62 blocks of 16 ports per stage
MAX_TP = REPLICA_STRIDE - 1                        # the control port + 15 data ports


def base() -> int:
    return int(os.getenv("CONNEX_PP_PORT_BASE", "47000"))


def control_port(stage: int, replica: int, port_base: Optional[int] = None) -> int:
    if stage < 0 or not 0 <= replica < MAX_REPLICAS:
        raise ValueError(f"stage {stage} / replica {replica} out of range (replica < {MAX_REPLICAS})")
    p = (base() if port_base is None else port_base) + STAGE_STRIDE * stage + REPLICA_STRIDE * replica
    if p + REPLICA_STRIDE > 65536:
        raise ValueError(f"stage {stage} replica {replica}: port {p} out of range (lower CONNEX_PP_PORT_BASE)")
    return p


def _check_tp(tp_rank: int) -> None:
    if not 0 <= tp_rank < MAX_TP:
        raise ValueError(f"TP rank {tp_rank} out of range (< {MAX_TP})")


def data_port(stage: int, replica: int, tp_rank: int = 0, port_base: Optional[int] = None) -> int:
    _check_tp(tp_rank)
    return control_port(stage, replica, port_base) + 1 + tp_rank


def rank_port(rank0_port: int, tp_rank: int) -> int:
    """Data port of ``tp_rank`` given TP rank 0's (0 stays 0: ephemeral)."""
    if not rank0_port:
        return 0
    _check_tp(tp_rank)
    return rank0_port + tp_rank


def main(argv: List[str]) -> int:
    if len(argv) not in (3, 4) or argv[0] not in ("control", "data"):
        print("usage: python -m connex.adapters.vllm.pp.ports control|data STAGE REPLICA [TP_RANK]", file=sys.stderr)
        return 2
    stage, replica = int(argv[1]), int(argv[2])
    print(control_port(stage, replica) if argv[0] == "control" else
          data_port(stage, replica, int(argv[3]) if len(argv) > 3 else 0))
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
