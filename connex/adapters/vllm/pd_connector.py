"""``ConnexConnector``: prefill-decode disaggregation for upstream vLLM's
KV-connector API (reference ``connex/adapters/vllm/pd_connector.py``).

    vllm serve <model> --kv-transfer-config '{"kv_connector": "ConnexConnector",
        "kv_connector_module_path": "connex.adapters.vllm.pd_connector",
        "kv_role": "kv_producer",                   # "kv_consumer" on decode
        "kv_connector_extra_config": {"ctrl_port": 17100}}'

Pull based, on :mod:`connex.pd.transfer`:

1. the PD router sends the prompt to a prefill instance with
   ``kv_transfer_params={"do_remote_decode": true, "transfer_id": T}``; when
   the request finishes the scheduler keeps its blocks and answers with
   ``kv_transfer_params`` naming ``T``, the control address and the prompt
   length; the worker *holds* the blocks under ``T`` (a lease renewed by
   each acquire, expiring after ``retain_s``);
2. the decode instance reports the prompt as externally computed (async
   load); its worker acquires ``T`` and reads the blocks one-sidedly (NVLink
   peer mappings inside a box, the native engine across hosts) and reports
   the request received; a failed read becomes load errors for its blocks;
3. when the decode request finishes, its worker releases ``T``; a decode
   that died instead leaves the hold for a re-pull by the next decode
   instance.

``kv_connector_extra_config``: ``backend`` (``auto`` | ``nvlink`` | ``cxengine``
| ``loopback``), ``host``, ``ctrl_port`` (TP rank r uses ``ctrl_port + r``),
``bind_ip``, ``retain_s`` (default 60), ``release`` (``on_finish`` |
``after_pull``).  Equal TP sizes on both sides (rank r reads rank r).
"""
from __future__ import annotations

import logging
import os
import uuid
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Tuple

import torch
from vllm.distributed.kv_transfer.kv_connector.v1.base import (KVConnectorBase_V1, KVConnectorMetadata,
                                                               KVConnectorRole)

log = logging.getLogger("connex.vllm.pd")


@dataclass
class ConnexConnectorMetadata(KVConnectorMetadata):
    load: Dict[str, Tuple[str, str, List[int], int]] = field(default_factory=dict)   # req -> (ctrl, T, blocks, n)
    hold: Dict[str, Tuple[str, List[int]]] = field(default_factory=dict)             # req -> (T, blocks)
    release: List[Tuple[str, str]] = field(default_factory=list)                      # (ctrl, T)


def _extra(vllm_config) -> dict:
    return dict(getattr(vllm_config.kv_transfer_config, "kv_connector_extra_config", None) or {})


def _tp_rank() -> int:
    try:
        from vllm.distributed.parallel_state import get_tensor_model_parallel_rank
        return get_tensor_model_parallel_rank()
    except Exception:  # noqa: BLE001 - not initialised (tests, scheduler process)
        return 0


def _host(extra: dict) -> str:
    return extra.get("host") or os.getenv("CONNEX_HOST_IP") or os.getenv("VLLM_HOST_IP") or "127.0.0.1"


def _ctrl_for_rank(ctrl: str, rank: int) -> str:
    host, port = ctrl.rsplit(":", 1)
    return f"{host}:{int(port) + rank}"


class ConnexConnector(KVConnectorBase_V1):
    def __init__(self, vllm_config, role: KVConnectorRole, kv_cache_config=None):
        super().__init__(vllm_config, role, kv_cache_config)
        tc = vllm_config.kv_transfer_config
        self.extra = _extra(vllm_config)
        self.kv_role = getattr(tc, "kv_role", "kv_both")
        self.ctrl_port = int(self.extra.get("ctrl_port") or getattr(tc, "kv_port", 0) or 17100)
        self.host = _host(self.extra)
        self.block_size = int(getattr(getattr(vllm_config, "cache_config", None), "block_size", 16) or 16)
        # scheduler side
        self._to_load: Dict[str, Tuple[str, str, List[int], int]] = {}
        self._to_hold: Dict[str, Tuple[str, List[int]]] = {}
        self._to_release: List[Tuple[str, str]] = []
        self._loaded: set = set()
        # worker side
        self.producer = None
        self.consumer = None
        self._load_blocks: Dict[str, List[int]] = {}
        self._load_errors: set = set()

    # ================================================================ scheduler
    def get_num_new_matched_tokens(self, request, num_computed_tokens: int):
        p = request.kv_transfer_params or {}
        if not p.get("do_remote_prefill") or request.request_id in self._loaded:
            return 0, False
        n = min(int(p.get("remote_num_tokens", len(request.prompt_token_ids))), len(request.prompt_token_ids))
        count = n - num_computed_tokens
        return (count, True) if count > 0 else (0, False)

    def update_state_after_alloc(self, request, blocks, num_external_tokens: int):
        p = request.kv_transfer_params or {}
        if num_external_tokens <= 0 or not p.get("do_remote_prefill") or request.request_id in self._loaded:
            return
        ids = list(blocks.get_block_ids()[0])
        self._to_load[request.request_id] = (p["remote_ctrl"], p["transfer_id"], ids, num_external_tokens)
        self._loaded.add(request.request_id)

    def build_connector_meta(self, scheduler_output) -> KVConnectorMetadata:
        meta = ConnexConnectorMetadata(load=self._to_load, hold=self._to_hold, release=self._to_release)
        self._to_load, self._to_hold, self._to_release = {}, {}, []
        return meta

    def request_finished(self, request, block_ids) -> Tuple[bool, Optional[Dict[str, Any]]]:
        p = request.kv_transfer_params or {}
        self._loaded.discard(request.request_id)
        if p.get("do_remote_decode"):                 # a prefill: keep the blocks for the decode side
            tid = p.get("transfer_id") or uuid.uuid4().hex
            ids = list(block_ids[0] if block_ids and isinstance(block_ids[0], (list, tuple)) else block_ids)
            self._to_hold[request.request_id] = (tid, ids)
            return True, {"do_remote_prefill": True, "do_remote_decode": False, "transfer_id": tid,
                          "remote_ctrl": f"{self.host}:{self.ctrl_port}",
                          "remote_num_tokens": len(request.prompt_token_ids)}
        if p.get("do_remote_prefill") and self.extra.get("release", "on_finish") == "on_finish":
            self._to_release.append((p["remote_ctrl"], p["transfer_id"]))
        return False, None

    # ================================================================== worker
    def register_kv_caches(self, kv_caches: Dict[str, torch.Tensor]):
        from connex.pd.dataplane import make_plane
        from connex.pd.kv_layout import tensor_layout
        from connex.pd.transfer import KVConsumer, KVProducer
        tensors = list(kv_caches.values())
        nb = getattr(self._kv_cache_config, "num_blocks", None) or _guess_blocks(tensors[0])
        layouts = [tensor_layout(t, nb) for t in tensors]
        rank = _tp_rank()
        dev = tensors[0].device
        self.plane = make_plane("vllm", 0 if self.kv_role == "kv_producer" else 1, 0, rank, ip=self.host,
                                backend=self.extra.get("backend"), device=dev.index if dev.type == "cuda" else None)
        if self.kv_role in ("kv_producer", "kv_both"):
            self.producer = KVProducer(self.plane, layouts, bind_ip=self.extra.get("bind_ip", "0.0.0.0"),
                                       port=self.ctrl_port + rank, retain_s=float(self.extra.get("retain_s", 60)),
                                       block_size=self.block_size, device=str(dev))
        if self.kv_role in ("kv_consumer", "kv_both"):
            self.consumer = KVConsumer(self.plane, layouts, block_size=self.block_size,
                                       release_after_pull=self.extra.get("release") == "after_pull",
                                       device=str(dev), register=self.producer is None)
        self.rank = rank

    def start_load_kv(self, forward_context, **kwargs) -> None:
        if not self.has_connector_metadata():
            return
        meta: ConnexConnectorMetadata = self._get_connector_metadata()
        for req_id, (tid, blocks) in meta.hold.items():
            if self.producer is not None:
                self.producer.hold(req_id, tid, blocks)
        for ctrl, tid in meta.release:
            if self.consumer is not None:
                self.consumer.release(_ctrl_for_rank(ctrl, self.rank), tid)
        for req_id, (ctrl, tid, blocks, n) in meta.load.items():
            need = -(-n // self.block_size)
            self._load_blocks[req_id] = blocks[:need]
            self.consumer.pull(req_id, _ctrl_for_rank(ctrl, self.rank), tid, blocks[:need])

    def wait_for_layer_load(self, layer_name: str) -> None:
        return          # whole-request pulls finish before the request is scheduled (async load)

    def save_kv_layer(self, layer_name: str, kv_layer, attn_metadata, **kwargs) -> None:
        return          # pull based: the decode side reads

    def wait_for_save(self):
        return

    def get_finished(self, finished_req_ids):
        sending = set(self.producer.take_finished()) if self.producer is not None else set()
        recving = set()
        if self.consumer is not None:
            for r in self.consumer.take_done():
                recving.add(r.req_id)
                if not r.ok:
                    log.warning("KV pull of %s failed: %s", r.req_id, r.why)
                    self._load_errors.update(self._load_blocks.get(r.req_id, []))
                self._load_blocks.pop(r.req_id, None)
        return (sending or None), (recving or None)

    def get_block_ids_with_load_errors(self) -> set:
        out, self._load_errors = self._load_errors, set()
        return out

    def shutdown(self):
        for x in (self.consumer, self.producer):
            if x is not None:
                x.close()
        if getattr(self, "plane", None) is not None:
            self.plane.close()


def _guess_blocks(t: torch.Tensor) -> int:
    return t.shape[1] if t.dim() >= 5 and t.shape[0] == 2 else t.shape[0]
