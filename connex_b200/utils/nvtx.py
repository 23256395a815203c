"""NVTX ranges around the runtime's phases, on with ``CONNEX_NVTX=1``.

The ranges name what a device timeline or an ``ncu --nvtx --nvtx-include``
filter needs to tell apart: prefill / decode and their layers, the layerwise
KV push, the EP layer's phases (count, dispatch, gate/up, down, combine) and
the weight broadcast.  When the variable is unset every call is a branch on a
module constant (no NVTX call, nothing recorded).
"""
from __future__ import annotations

import os
from contextlib import contextmanager

ON = os.getenv("CONNEX_NVTX", "0") == "1"


def push(name: str) -> None:
    if ON:
        import torch
        torch.cuda.nvtx.range_push(name)


def pop() -> None:
    if ON:
        import torch
        torch.cuda.nvtx.range_pop()


@contextmanager
def nvtx_range(name: str):
    push(name)
    try:
        yield
    finally:
        pop()
