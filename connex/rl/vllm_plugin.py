"""vLLM general plugin: registers the ``connex`` weight-transfer backend in
every vLLM process (reference ``connex/rl/vllm_plugin.py``)."""


def register():
    try:
        from .vllm_backend import register as _register
    except ImportError:   # a vLLM without the pluggable weight-transfer API
        return
    _register()
