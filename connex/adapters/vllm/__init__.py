"""vLLM adapters: the ``ConnexConnector`` KV connector (``pd_connector``) and
the general-plugin registration (``plugin``)."""
