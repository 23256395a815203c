"""vLLM general plugin: registers ``ConnexConnector`` with vLLM's KV-connector
factory in every vLLM process (reference ``connex/adapters/vllm/plugin.py``)."""


def register() -> None:
    try:
        from vllm.distributed.kv_transfer.kv_connector.factory import KVConnectorFactory
    except ImportError:     # a vLLM without the v1 connector API
        return
    if "ConnexConnector" not in KVConnectorFactory._registry:
        KVConnectorFactory.register_connector("ConnexConnector", "connex.adapters.vllm.pd_connector",
                                              "ConnexConnector")
