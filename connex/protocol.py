"""Stable logical endpoint identity (LID).

A LID names a role in the serving system -- ``(model, stage, shard, replica)``
plus an optional prefill/decode role -- independently of the process and
address that currently plays it.  Addresses, liveness and state can change;
the LID stays.  Mirrors ``connex/protocol.py:10-71`` of the reference: a
LID compares equal to its 5-tuple and, ignoring the PD role, to a 4-tuple.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Tuple


class PDRole:
    """Prefill/decode roles of a PD-disaggregated deployment."""

    NONE = "none"
    PREFILL = "prefill"
    DECODE = "decode"


@dataclass
class LogicalEndpointID:
    model_name: str
    stage_idx: int
    shard_idx: int = 0
    replica_idx: int = 0
    pd_role: str = PDRole.NONE

    def to_tuple(self) -> Tuple[str, int, int, int, str]:
        return (self.model_name, self.stage_idx, self.shard_idx, self.replica_idx, self.pd_role)

    def __hash__(self) -> int:
        return hash(self.to_tuple())

    def __eq__(self, other: object) -> bool:
        if isinstance(other, LogicalEndpointID):
            return self.to_tuple() == other.to_tuple()
        if isinstance(other, tuple):
            mine = self.to_tuple()
            return mine[:4] == other if len(other) == 4 else mine == other
        return False

    @property
    def is_decode(self) -> bool:
        return self.pd_role == PDRole.DECODE

    @property
    def is_pd_mode(self) -> bool:
        return self.pd_role != PDRole.NONE

    def __str__(self) -> str:
        base = f"LID({self.model_name}:s{self.stage_idx}:sh{self.shard_idx}:r{self.replica_idx}"
        return base + (")" if self.pd_role == PDRole.NONE else f":{self.pd_role})")

    __repr__ = __str__
