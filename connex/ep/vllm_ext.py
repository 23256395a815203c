"""vLLM glue for ``connex.ep`` (upstream vLLM, no fork; written against the
``EplbState`` layout of vLLM 0.22).

Worker side: start vLLM with ``--enable-expert-parallel --enable-eplb
--worker-extension-cls connex.ep.vllm_ext.ConnexEPWorker`` (and an EPLB
``step_interval`` longer than the run: Connex owns the map).  The controller
reaches the ``connex_ep_*`` methods through vLLM's ``/collective_rpc``
(``VLLM_SERVER_DEV_MODE=1``); vLLM runs them on every worker between two
engine steps, which is the cut-over point an epoch needs.  The methods are
those of :class:`connex.ep.engine_ext.EPWorkerCore`; this module supplies the
engine hooks: vLLM's per-model ``EplbModelState`` holds
``physical_to_logical_map [L, P]``, ``logical_to_physical_map [L, E, W]`` and
``logical_replica_count [L, E]``, and the MoE layers hand out their expert
weights with ``get_expert_weights()`` (reference
``connex/ep/vllm_ext.py:139-338``).

EPLB needs a model implementing vLLM's ``MixtureOfExperts`` interface;
:func:`enable_olmoe_eplb` adds it to OLMoE when the installed vLLM lacks it
(reference ``connex/ep/vllm_ext.py:47-110``).  The ``connex_ep`` plugin
applies it only with ``CONNEX_EP=1``.

Controller side: :class:`VLLMEPEngine` (``EPController`` engine handle for
one vLLM server, all EP ranks).
"""
from __future__ import annotations

import logging
import os
import sys

from connex.ep.engine_ext import EngineMaps, EPWorkerCore, HTTPEPEngine, slot_sums

log = logging.getLogger("connex.ep")

_olmoe_done = False

_slot_sums = slot_sums          # the reference's private name for the checksum helper


def register() -> None:
    """``vllm.general_plugins`` entry point; opt-in with ``CONNEX_EP=1``."""
    if os.environ.get("CONNEX_EP", "").lower() in ("1", "true", "yes"):
        enable_olmoe_eplb()


def enable_olmoe_eplb() -> bool:
    """Give vLLM's ``OlmoeForCausalLM`` the ``MixtureOfExperts`` interface
    (idempotent; False without vLLM or when the model has it already)."""
    global _olmoe_done
    if _olmoe_done:
        return True
    try:
        from vllm.model_executor.models import olmoe
        from vllm.model_executor.models.interfaces import MixtureOfExperts
        from vllm.model_executor.models.registry import ModelRegistry
    except ImportError:
        return False
    _olmoe_done = True
    if hasattr(olmoe.OlmoeForCausalLM, "set_eplb_state"):
        return False
    # OLMoE builds its experts without the EPLB arguments: pass them when EPLB is on
    # (the module names its MoE constructor FusedMoE in 0.22, FusedMoEFactory elsewhere)
    for ctor_name in ("FusedMoEFactory", "FusedMoE"):
        ctor = getattr(olmoe, ctor_name, None)
        if ctor is None:
            continue

        def with_eplb(*a, _ctor=ctor, **kw):
            from vllm.config import get_current_vllm_config
            pc = get_current_vllm_config().parallel_config
            if pc.enable_eplb:
                kw.setdefault("enable_eplb", True)
                kw.setdefault("num_redundant_experts", pc.eplb_config.num_redundant_experts)
            return _ctor(*a, **kw)
        setattr(olmoe, ctor_name, with_eplb)
        break

    class OlmoeForCausalLM(olmoe.OlmoeForCausalLM, MixtureOfExperts):
        def __init__(self, *, vllm_config, prefix=""):
            super().__init__(vllm_config=vllm_config, prefix=prefix)
            hf = vllm_config.model_config.hf_config
            pc = vllm_config.parallel_config
            extra = pc.eplb_config.num_redundant_experts if pc.enable_eplb else 0
            self.moe_layers = [l.mlp.experts for l in self.model.layers
                               if isinstance(getattr(l, "mlp", None), olmoe.OlmoeMoE)]
            self.expert_weights = []
            self.num_moe_layers = len(self.moe_layers)
            self.num_expert_groups = 1
            self.num_shared_experts = 0
            self.num_logical_experts = self.num_routed_experts = hf.num_experts
            self.num_redundant_experts = extra
            self.num_physical_experts = hf.num_experts + extra
            self.num_local_physical_experts = getattr(self.moe_layers[0], "local_num_experts",
                                                      self.num_physical_experts)

        def update_physical_experts_metadata(self, num_physical_experts, num_local_physical_experts):
            self.num_physical_experts = num_physical_experts
            self.num_local_physical_experts = num_local_physical_experts
            self.num_redundant_experts = num_physical_experts - self.num_logical_experts
            for layer in self.moe_layers:
                layer.update_expert_map()

    olmoe.OlmoeForCausalLMEP = OlmoeForCausalLM
    ModelRegistry.register_model("OlmoeForCausalLM", OlmoeForCausalLM)
    return True


# A vLLM worker imports this module (its extension class) before it builds
# the model, so choosing the extension is the opt-in.  A controller process
# that only needs VLLMEPEngine has not imported vLLM and does not load it here.
if "vllm" in sys.modules:
    enable_olmoe_eplb()


class ConnexEPWorker(EPWorkerCore):
    """Mixed into vLLM's GPU worker (``--worker-extension-cls``)."""

    def _eplb_model(self):
        st = getattr(self.model_runner, "eplb_state", None)
        if st is None or not st.model_states:
            raise RuntimeError("EPLB is off: start vLLM with --enable-expert-parallel --enable-eplb")
        return next(iter(st.model_states.values()))

    def _ep_rank(self) -> int:
        from vllm.distributed import get_ep_group
        return get_ep_group().rank_in_group

    def _ep_maps(self) -> EngineMaps:
        from vllm.distributed import get_ep_group
        ms = self._eplb_model()
        R = get_ep_group().world_size
        P = ms.physical_to_logical_map.shape[1]
        return EngineMaps(ms.physical_to_logical_map, ms.logical_to_physical_map, ms.logical_replica_count,
                          num_ranks=R, slots_per_rank=P // R, num_experts=ms.model.num_logical_experts)

    def _expert_layers(self) -> list:
        return [list(layer.get_expert_weights()) for layer in self._eplb_model().model.moe_layers]

    def _ep_load_counts(self):
        w = getattr(self._eplb_model(), "expert_load_window", None)
        return None if w is None else w.sum(dim=0).sum(dim=0).cpu().tolist()


class VLLMEPEngine(HTTPEPEngine):
    """``EPController`` engine handle for one vLLM server: POST
    ``/collective_rpc`` (``VLLM_SERVER_DEV_MODE=1``), one result per worker."""

    path = "/collective_rpc"


__all__ = ["register", "enable_olmoe_eplb", "ConnexEPWorker", "VLLMEPEngine"]
