"""SGLang adapters.

* ``connex.adapters.sglang.pd_backend`` -- the ``connex`` KV transfer backend
  for SGLang prefill-decode disaggregation (plugin entry point ``connex``).
* ``connex.ep.sglang_ext`` -- the EP control path (plugin entry point
  ``connex_ep``).

Importing this package does not import SGLang.
"""
