"""SGLang adapters.

* :class:`ConnexPPGroup` / :func:`make_pp_group` -- a ``GroupCoordinator``-
  compatible ``pp_group`` over the Connex step protocol (external elastic PP,
  communication side);
* ``connex.adapters.sglang.pd_backend`` -- the ``connex`` KV transfer backend
  for SGLang prefill-decode disaggregation (plugin entry point ``connex``);
* ``connex.ep.sglang_ext`` -- the EP control path (plugin entry point
  ``connex_ep``).

Importing this package does not import SGLang.
"""
from connex.adapters.sglang.pp_group import MISSING_HERE, MSG_TYPE, REPREFILLED, ConnexPPGroup  # noqa: F401
from connex.adapters.sglang.setup import make_pp_group  # noqa: F401

__all__ = ["ConnexPPGroup", "make_pp_group", "MSG_TYPE", "MISSING_HERE", "REPREFILLED"]
