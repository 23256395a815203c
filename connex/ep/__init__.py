"""Expert parallelism with recovery and elasticity (reference ``connex/ep``).

* :class:`PlacementTable` -- versioned expert placement (slots, replicas,
  rank states, routable masks, repair planning);
* :class:`ExpertStore` -- one rank's expert weights, readable by peers
  (CUDA IPC + the ``copy_segments`` kernel inside an NVLink box, one-sided
  transport reads otherwise);
* :class:`EPController` -- every change in two epochs (route around, copy,
  route to the new copies).

Engine glue: ``connex.ep.vllm_ext`` (vLLM worker extension) and
``connex.ep.sglang_ext`` (SGLang scheduler control path); this build's own
fused EP layer is ``connex_b200.parallel.ep.EPMoE``.
"""
from connex.ep.placement import (DOWN, DRAINING, UP, Move, PlacementError, PlacementTable,  # noqa: F401
                                 logical_to_physical)
from connex.ep.mover import ExpertStore, moves_by_rank  # noqa: F401
from connex.ep.controller import EPController, LocalEngine  # noqa: F401

__all__ = ["PlacementTable", "Move", "PlacementError", "logical_to_physical", "UP", "DRAINING", "DOWN",
           "ExpertStore", "moves_by_rank", "EPController", "LocalEngine"]
