"""Engine adapters (vLLM / SGLang plugin shims) over the connex libraries;
each imports its engine only when loaded by that engine."""
