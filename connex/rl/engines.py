"""Rollout instances backed by engine servers over HTTP (reference
``connex/rl/engines.py:30-161``).

* :class:`VLLMInstance` -- ``vllm serve`` with the ``connex`` weight-transfer
  backend (:mod:`connex.rl.vllm_backend`) and its RL routes enabled; an
  update is ``/init_weight_transfer_engine`` (once), then
  ``/start_weight_update``, ``/update_weights``, ``/finish_weight_update``.
* :class:`SGLangInstance` -- an SGLang server started with
  ``--custom-weight-loader connex.rl.sglang_ext.connex_load``; an update is
  ``/update_weights_from_tensor`` carrying the control record.

Both generate from token ids.  A transport error or non-200 reply is
:class:`InstanceDead`; ``finish_reason == "abort"`` is :class:`Aborted`.
"""
from __future__ import annotations

import asyncio
import base64
import io
import json
import pickle

from .rollout import Aborted, InstanceDead, RolloutInstance
from .sglang_ext import LOADER, control_payload


class _HTTPInstance(RolloutInstance):
    def __init__(self, name, url, model, registry_url, member=None, timeout=600):
        self.name = name
        self.url = url.rstrip("/")
        self.model = model
        self.registry_url = registry_url
        self.member = member or name
        self.version = None
        self.timeout = timeout
        self._session = None

    async def _client(self):
        import aiohttp
        if self._session is None or self._session.closed:
            # idle connections shorter than typical server keep-alive (5 s), so a
            # pooled connection the server already closed is never reused
            self._session = aiohttp.ClientSession(
                timeout=aiohttp.ClientTimeout(total=self.timeout), trust_env=False,
                connector=aiohttp.TCPConnector(keepalive_timeout=2.0, limit=0))
        return self._session

    async def _post(self, path, body=None, params=None, allow_404=False):
        import aiohttp
        s = await self._client()
        for attempt in (0, 1):
            try:
                async with s.post(self.url + path, json=body, params=params) as r:
                    data = await r.read()
                    if allow_404 and r.status == 404:
                        return None
                    if r.status != 200:
                        raise InstanceDead(f"{path}: HTTP {r.status}: {data[:300]!r}")
                    return data
            except aiohttp.ServerDisconnectedError as e:
                if attempt:     # a dead server also refuses the retry's fresh connection
                    raise InstanceDead(f"{path}: {e!r}") from e
            except (aiohttp.ClientError, asyncio.TimeoutError, OSError) as e:
                raise InstanceDead(f"{path}: {e!r}") from e

    async def close(self):
        if self._session is not None:
            await self._session.close()


class VLLMInstance(_HTTPInstance):
    """``req``: ``{"prompt_ids", "max_tokens", "temperature", "seed"}``."""

    _inited = False

    async def generate(self, req, partial=None):
        body = {"model": self.model, "prompt": list(req["prompt_ids"]) + list(partial or []),
                "max_tokens": req["max_tokens"] - len(partial or []), "temperature": req.get("temperature", 0.0),
                "seed": req.get("seed"), "ignore_eos": req.get("ignore_eos", False), "logprobs": 0,
                "return_tokens_as_token_ids": True}
        ch = json.loads(await self._post("/v1/completions", body))["choices"][0]
        if ch.get("finish_reason") == "abort":
            raise Aborted()
        toks = ch.get("token_ids")
        if toks is None:
            toks = [int(t.split(":", 1)[1]) for t in ch["logprobs"]["tokens"]]
        return {"tokens": toks, "finish_reason": ch.get("finish_reason")}

    async def abort_all(self):
        await self._post("/pause", params={"mode": "abort", "clear_cache": "false"})
        await self._post("/resume")

    async def update(self, version):
        if not self._inited:
            await self._post("/init_weight_transfer_engine",
                             {"init_info": {"registry_url": self.registry_url, "member": self.member}})
            self._inited = True
        await self._post("/start_weight_update")
        await self._post("/update_weights", {"update_info": {"version": version}})
        await self._post("/finish_weight_update", {"weight_version": str(version)})
        self.version = version


class SGLangInstance(_HTTPInstance):
    def __init__(self, *a, tp_size: int = 1, **kw):
        super().__init__(*a, **kw)
        self.tp_size = tp_size

    async def generate(self, req, partial=None):
        sp = {"max_new_tokens": req["max_tokens"], "temperature": req.get("temperature", 0.0),
              "ignore_eos": req.get("ignore_eos", False)}
        if req.get("seed") is not None:
            sp["sampling_seed"] = req["seed"]
        out = json.loads(await self._post("/generate", {"input_ids": list(req["prompt_ids"]), "sampling_params": sp}))
        meta = out.get("meta_info") or {}
        fr = meta.get("finish_reason") or {}
        if isinstance(fr, dict) and fr.get("type") == "abort":
            raise Aborted()
        return {"tokens": out["output_ids"], "finish_reason": fr, "weight_version": meta.get("weight_version")}

    async def abort_all(self):
        await self._post("/abort_request", {"abort_all": True})

    def payload(self, version):
        buf = io.BytesIO()
        pickle.dump(control_payload(self.registry_url, version, self.member), buf)
        return [base64.b64encode(buf.getvalue()).decode()] * self.tp_size

    async def update(self, version):
        await self._post("/begin_weight_update", {}, allow_404=True)   # newer servers only
        await self._post("/update_weights_from_tensor", {
            "serialized_named_tensors": self.payload(version), "load_format": LOADER, "flush_cache": True,
            "weight_version": str(version)})
        await self._post("/end_weight_update", {}, allow_404=True)
        self.version = version
