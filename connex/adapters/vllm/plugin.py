"""vLLM general plugin: registers ``ConnexConnector`` with vLLM's KV-connector
factory in every vLLM process (reference ``connex/adapters/vllm/plugin.py``)
and, with ``CONNEX_PP_GROUP=1``, wraps each worker's pipeline group in
:class:`connex.adapters.vllm.pp.group.ConnexPPGroup` right after vLLM creates
its model-parallel groups."""
import functools
import os


def _wrap_pp_groups() -> None:
    from vllm.distributed import parallel_state as ps
    orig = ps.initialize_model_parallel
    if getattr(orig, "_connex_pp", False):
        return

    @functools.wraps(orig)
    def initialize_model_parallel(*a, **k):
        out = orig(*a, **k)
        from connex.adapters.vllm.pp.group import install
        install()
        return out
    initialize_model_parallel._connex_pp = True
    ps.initialize_model_parallel = initialize_model_parallel


def register() -> None:
    if os.getenv("CONNEX_PP_GROUP") == "1":
        try:
            _wrap_pp_groups()
        except ImportError:
            pass
    try:
        from vllm.distributed.kv_transfer.kv_connector.factory import KVConnectorFactory
    except ImportError:     # a vLLM without the v1 connector API
        return
    if "ConnexConnector" not in KVConnectorFactory._registry:
        KVConnectorFactory.register_connector("ConnexConnector", "connex.adapters.vllm.pd_connector",
                                              "ConnexConnector")
