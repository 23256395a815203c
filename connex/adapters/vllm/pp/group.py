"""``ConnexPPGroup`` for upstream vLLM, in-process pipeline mode (reference
``connex/adapters/vllm/pp/group.py``).

vLLM's workers reach their pipeline neighbours through the PP
``GroupCoordinator`` (``get_pp_group()``): ``isend_tensor_dict`` /
``irecv_tensor_dict`` (hidden states and residual going forward,
``vllm/v1/worker/gpu_worker.py``), their blocking forms, and broadcasts of
sampled tokens / logits from the last rank.  :class:`ConnexPPGroup` wraps
vLLM's own coordinator and moves only the forward tensor dicts:

* the metadata (keys, dtypes, shapes, and any non-tensor or CPU values) goes
  through the wrapped coordinator's ``send_object`` / ``recv_object`` (its
  CPU group), so it stays ordered with everything else vLLM sends;
* the GPU tensors go over a per-(pipeline rank, TP rank) link of this
  framework: the GPU-driven channel (:class:`connex_b200.parallel.p2pchan.
  ChanLinks`: a ring in the receiver's HBM written over NVLink by a copy
  kernel, ready/credit counters, bounded waits) by default, or elastic NCCL
  pair links (:class:`connex_b200.parallel.pplink.PairLinks`, also on gloo
  for CPU runs).  Each TP rank sends its whole tensors to the same TP rank of
  the next stage, so vLLM's all-gather slicing is not used.

Everything else (``broadcast_tensor_dict``, ``device_group``, ranks, ...) is
the wrapped coordinator's.  :func:`install` swaps the group into vLLM's
``parallel_state`` inside a worker (``CONNEX_PP_GROUP=1`` makes the vLLM
general plugin do it when the model parallel groups exist).
"""
from __future__ import annotations

import logging
import os
from collections import Counter
from typing import Any, Callable, List, Optional, Tuple

log = logging.getLogger("connex.adapters.vllm.pp")

_TENSOR = "__cx_tensor__"


class ConnexPPGroup:
    def __init__(self, base, links=None, *, tp_rank: int = 0, store=None, device=None, kind: Optional[str] = None):
        self._base = base
        self.tp_rank = tp_rank
        self.me = self.name(base.rank_in_group)
        if links is None:
            links = self._make_links(store, device, kind or os.getenv("CONNEX_PP_GROUP_LINKS", "chan"))
        self.links = links
        self.stats: Counter = Counter()

    def name(self, pp_rank: int) -> str:
        return f"cxvpp{pp_rank}.tp{self.tp_rank}"

    def _make_links(self, store, device, kind: str):
        import torch
        import torch.distributed as dist
        if store is None:
            store = dist.distributed_c10d._get_default_store()
        dev = torch.device(device) if device is not None else (
            torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu"))
        if kind == "chan" and dev.type == "cuda":
            from connex_b200.parallel.p2pchan import ChanLinks
            return ChanLinks(dist.PrefixStore("cxvpp-chan/", store), self.me, dev)
        from connex_b200.parallel.pplink import PairLinks
        return PairLinks(dist.PrefixStore("cxvpp-nccl/", store), self.me, dev)

    def __getattr__(self, item):
        # only reached for attributes this wrapper does not define
        return getattr(self._base, item)

    # ------------------------------------------------------------------ metadata
    def _split(self, tensor_dict: dict) -> Tuple[list, list]:
        """Tensors on the links' device go over the link; anything else rides in the metadata."""
        import torch
        meta, dev = [], []
        for k, v in tensor_dict.items():
            if isinstance(v, torch.Tensor) and v.device.type == self.links.device.type:
                meta.append((k, (_TENSOR, str(v.dtype).replace("torch.", ""), tuple(v.shape))))
                dev.append(v.contiguous())
            else:
                meta.append((k, v))
        return meta, dev

    # ------------------------------------------------------------------ sends
    def isend_tensor_dict(self, tensor_dict: dict, dst: Optional[int] = None, all_gather_group: Any = None,
                          all_gather_tensors: Optional[dict] = None) -> list:
        if self._base.world_size <= 1:
            return []
        if dst is None:
            dst = (self._base.rank_in_group + 1) % self._base.world_size
        meta, dev = self._split(tensor_dict)
        self._base.send_object(meta, dst=dst)
        if dev:
            self.links.open_tx(self.name(dst)).send(dev)
        self.stats["sent"] += 1
        self.stats["sent_tensors"] += len(dev)
        return []

    def send_tensor_dict(self, tensor_dict: dict, dst: Optional[int] = None, all_gather_group: Any = None,
                         all_gather_tensors: Optional[dict] = None):
        self.isend_tensor_dict(tensor_dict, dst, all_gather_group, all_gather_tensors)
        return None

    # ------------------------------------------------------------------ receives
    def irecv_tensor_dict(self, src: Optional[int] = None, all_gather_group: Any = None,
                          all_gather_tensors: Optional[dict] = None
                          ) -> Tuple[Optional[dict], List[Any], List[Callable[[], None]]]:
        import torch
        if self._base.world_size <= 1:
            return None, [], []
        if src is None:
            src = (self._base.rank_in_group - 1) % self._base.world_size
        meta = self._base.recv_object(src=src)
        out, bufs = {}, []
        dev = self.links.device
        for k, v in meta:
            if isinstance(v, tuple) and len(v) == 3 and v[0] == _TENSOR:
                t = torch.empty(v[2], dtype=getattr(torch, v[1]), device=dev)
                out[k] = t
                bufs.append(t)
            else:
                out[k] = v
        post: List[Callable[[], None]] = []
        if bufs:
            link = self.links.open_rx(self.name(src))
            link.recv(bufs)
            ev = link.done_event()
            if ev is not None:
                post.append(lambda: torch.cuda.current_stream(dev).wait_event(ev))
        self.stats["received"] += 1
        return out, [], post

    def recv_tensor_dict(self, src: Optional[int] = None, all_gather_group: Any = None,
                         all_gather_tensors: Optional[dict] = None) -> Optional[dict]:
        td, handles, post = self.irecv_tensor_dict(src, all_gather_group, all_gather_tensors)
        for h in handles:
            h.wait()
        for fn in post:
            fn()
        return td

    def destroy(self) -> None:
        try:
            self.links.close()
        finally:
            destroy = getattr(self._base, "destroy", None)
            if destroy is not None:
                destroy()


def install(store=None, kind: Optional[str] = None) -> Optional[ConnexPPGroup]:
    """Wrap vLLM's PP group of this worker (after its model-parallel groups
    exist); a no-op without pipeline parallelism."""
    from vllm.distributed import parallel_state as ps
    base = getattr(ps, "_PP", None)
    if base is None or isinstance(base, ConnexPPGroup) or base.world_size <= 1:
        return base if isinstance(base, ConnexPPGroup) else None
    tp = getattr(ps, "_TP", None)
    grp = ConnexPPGroup(base, tp_rank=tp.rank_in_group if tp is not None else 0, store=store, kind=kind)
    ps._PP = grp
    log.info("vLLM PP group wrapped: %s, links %s", grp.me, type(grp.links).__name__)
    return grp


__all__ = ["ConnexPPGroup", "install"]
