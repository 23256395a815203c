"""connex: communication for distributed LLM serving in which the set of
peers keeps changing (reference ``connex/__init__.py``).

Endpoints are addressed by stable logical endpoint ids instead of ranks, so
they join, leave, fail and migrate while traffic is in flight.

* control plane: :mod:`connex.front_router` (client :mod:`connex.epc_client`)
  and the light :mod:`connex.directory`; mobility: :mod:`connex.elastic`;
* scenario libraries: :mod:`connex.pp`, :mod:`connex.pd`, :mod:`connex.ep`,
  :mod:`connex.rl`, :mod:`connex.agents`; serving: :mod:`connex.serving`;
* data plane: the native engine and the sm_100a kernels in ``connex_b200``.

Public names resolve lazily (PEP 562): ``import connex`` loads neither
torch nor the native extension.
"""

__version__ = "0.2.1"

_LAZY = {
    "DirectoryClient": ("connex.directory", "DirectoryClient"),
    "EndpointInfo": ("connex.directory", "EndpointInfo"),
    "ElasticPeerSet": ("connex.elastic", "ElasticPeerSet"),
    "LogicalEndpointID": ("connex.protocol", "LogicalEndpointID"),
    "PDRole": ("connex.protocol", "PDRole"),
    "EPCV2Client": ("connex.epc_client", "EPCV2Client"),
    "EPCV2ClientConfig": ("connex.epc_client", "EPCV2ClientConfig"),
    "EventType": ("connex.epc_client", "EventType"),
    "EPCV2TransportCapability": ("connex.epc_client", "TransportCapability"),
    "EPCV2RouteState": ("connex.epc_client", "RouteState"),
    "EPCV2LogicalEndpointID": ("connex.epc_client", "LogicalEndpointID"),
    "EPCV2RouteEntry": ("connex.epc_client", "RouteEntry"),
    "EPCV2Event": ("connex.epc_client", "Event"),
    "RouteTableCache": ("connex.epc_client", "RouteTableCache"),
    "DataPlaneManager": ("connex.epc_client", "DataPlaneManager"),
    "EPCV2ShadowConnectionManager": ("connex.epc_client", "ShadowConnectionManager"),
    "create_epc_client": ("connex.epc_client", "create_epc_client"),
}


def __getattr__(name):
    try:
        mod, attr = _LAZY[name]
    except KeyError:
        raise AttributeError(f"module 'connex' has no attribute {name!r}") from None
    import importlib
    value = getattr(importlib.import_module(mod), attr)
    globals()[name] = value
    return value


def __dir__():
    return sorted(set(globals()) | set(_LAZY))


__all__ = ["__version__", *_LAZY]
