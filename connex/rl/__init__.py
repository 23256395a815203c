"""Elastic, versioned weight synchronisation for RL post-training
(reference ``connex/rl/__init__.py``).

A trainer publishes version ``v`` (:class:`WeightPublisher`); rollout
engines pull it with one-sided reads (:class:`WeightSubscriber`) from the
trainer or from engines that already hold it (tree fan-out) and apply it in
one step; :class:`WeightRegistry` tracks members, the latest version and
its holders; :class:`RolloutPool` keeps each request on one version.
Inside one NVLink box, :mod:`connex_b200.parallel.wsync` broadcasts a
version to every GPU with one fused cast + relayout kernel instead.
"""
from .registry import RegistryClient, RegistryServer, WeightRegistry
from .rollout import InstanceState, RolloutInstance, RolloutPool
from .sync import WeightPublisher, WeightSubscriber
from .transport import EngineTransport, LocalTransport, NvlinkTransport, TransferError, make_transport
from .weights import WeightManifest, arena_size, pack_into, unpack

__all__ = ["WeightManifest", "pack_into", "unpack", "arena_size", "LocalTransport", "NvlinkTransport",
           "EngineTransport", "make_transport", "TransferError", "WeightRegistry", "RegistryServer",
           "RegistryClient", "WeightPublisher", "WeightSubscriber", "RolloutPool", "RolloutInstance",
           "InstanceState"]
