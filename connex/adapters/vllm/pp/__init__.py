"""Pieces of the external-PP deployment contract that do not depend on vLLM:
authenticated control frames (:mod:`.auth`), the port layout (:mod:`.ports`)
and per-step timestamps (:mod:`.trace`).  Importing needs neither torch nor
vLLM.  The stage-0 executor / stage server roles themselves are this
framework's own runtime (``connex.pp.link``, ``connex_b200.runtime.pp``)."""
