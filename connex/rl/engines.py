"""Rollout instances backed by engine servers over HTTP.

* :class:`VLLMInstance` -- ``vllm serve`` with the ``connex`` weight-transfer
  backend (:mod:`connex.rl.vllm_backend`) and its RL routes: an update is
  ``/init_weight_transfer_engine`` (first time only),
  ``/start_weight_update``, ``/update_weights``, ``/finish_weight_update``.
* :class:`SGLangInstance` -- an SGLang server started with
  ``--custom-weight-loader connex.rl.sglang_ext.connex_load``: an update is
  ``/update_weights_from_tensor`` carrying the pickled control record
  (bracketed by ``/begin_weight_update`` / ``/end_weight_update`` on servers
  that have them).

Both generate from token ids.  A transport error or a non-200 reply raises
:class:`InstanceDead`; a finish reason of ``abort`` raises :class:`Aborted`.
The routes and bodies are those engines' own APIs (reference
``connex/rl/engines.py:30-161`` drives the same ones).
"""
from __future__ import annotations

import asyncio
import base64
import json
import pickle
from typing import Any, List, Optional, Tuple

from .rollout import Aborted, InstanceDead, RolloutInstance
from .sglang_ext import LOADER, control_payload


class _Http:
    """A pooled aiohttp client for one server.  Idle connections expire after
    2 s -- below common server keep-alive (5 s) -- so a connection the server
    already closed is not reused; a disconnect is retried once on a fresh
    connection before it counts as a dead server."""

    def __init__(self, url: str, timeout: float):
        self.url = url.rstrip("/")
        self.timeout = timeout
        self._session = None

    async def _sess(self):
        import aiohttp
        if self._session is None or self._session.closed:
            self._session = aiohttp.ClientSession(
                timeout=aiohttp.ClientTimeout(total=self.timeout), trust_env=False,
                connector=aiohttp.TCPConnector(keepalive_timeout=2.0, limit=0))
        return self._session

    async def post(self, path: str, body: Any = None, params: Optional[dict] = None,
                   allow_404: bool = False) -> Optional[bytes]:
        import aiohttp
        session = await self._sess()
        last: Optional[BaseException] = None
        for _ in range(2):
            try:
                async with session.post(self.url + path, json=body, params=params) as r:
                    data = await r.read()
                    if r.status == 404 and allow_404:
                        return None
                    if r.status != 200:
                        raise InstanceDead(f"{path}: HTTP {r.status}: {data[:300]!r}")
                    return data
            except aiohttp.ServerDisconnectedError as e:
                last = e                          # maybe a stale pooled connection: once more
            except (aiohttp.ClientError, asyncio.TimeoutError, OSError) as e:
                raise InstanceDead(f"{path}: {e!r}") from e
        raise InstanceDead(f"{path}: {last!r}") from last

    async def close(self) -> None:
        if self._session is not None:
            await self._session.close()


class _HTTPInstance(RolloutInstance):
    def __init__(self, name, url, model, registry_url, member=None, timeout=600):
        self.name = name
        self.model = model
        self.registry_url = registry_url
        self.member = member or name
        self.version = None
        self.http = _Http(url, timeout)

    @property
    def url(self) -> str:
        return self.http.url

    async def _post(self, path, body=None, params=None, allow_404=False):
        return await self.http.post(path, body, params, allow_404)

    async def _run(self, steps: List[Tuple[str, Any, bool]]) -> None:
        for path, body, optional in steps:
            await self._post(path, body, allow_404=optional)

    async def close(self):
        await self.http.close()


class VLLMInstance(_HTTPInstance):
    """``req``: ``{"prompt_ids", "max_tokens", "temperature", "seed"}``."""

    _inited = False

    async def generate(self, req, partial=None):
        done = list(partial or [])
        body = {"model": self.model, "prompt": list(req["prompt_ids"]) + done,
                "max_tokens": req["max_tokens"] - len(done), "temperature": req.get("temperature", 0.0),
                "seed": req.get("seed"), "ignore_eos": req.get("ignore_eos", False), "logprobs": 0,
                "return_tokens_as_token_ids": True}
        choice = json.loads(await self._post("/v1/completions", body))["choices"][0]
        if choice.get("finish_reason") == "abort":
            raise Aborted()
        ids = choice.get("token_ids")
        if ids is None:                           # older servers: "token_id:<n>" strings in logprobs
            ids = [int(t.split(":", 1)[1]) for t in choice["logprobs"]["tokens"]]
        return {"tokens": ids, "finish_reason": choice.get("finish_reason")}

    async def abort_all(self):
        await self._post("/pause", params={"mode": "abort", "clear_cache": "false"})
        await self._post("/resume")

    async def update(self, version):
        steps = []
        if not self._inited:
            steps.append(("/init_weight_transfer_engine",
                          {"init_info": {"registry_url": self.registry_url, "member": self.member}}, False))
        steps += [("/start_weight_update", None, False),
                  ("/update_weights", {"update_info": {"version": version}}, False),
                  ("/finish_weight_update", {"weight_version": str(version)}, False)]
        await self._run(steps)
        self._inited = True
        self.version = version


class SGLangInstance(_HTTPInstance):
    def __init__(self, *a, tp_size: int = 1, **kw):
        super().__init__(*a, **kw)
        self.tp_size = tp_size

    async def generate(self, req, partial=None):
        sampling = {"max_new_tokens": req["max_tokens"], "temperature": req.get("temperature", 0.0),
                    "ignore_eos": req.get("ignore_eos", False)}
        if req.get("seed") is not None:
            sampling["sampling_seed"] = req["seed"]
        out = json.loads(await self._post("/generate", {"input_ids": list(req["prompt_ids"]),
                                                        "sampling_params": sampling}))
        meta = out.get("meta_info") or {}
        reason = meta.get("finish_reason") or {}
        if isinstance(reason, dict) and reason.get("type") == "abort":
            raise Aborted()
        return {"tokens": out["output_ids"], "finish_reason": reason, "weight_version": meta.get("weight_version")}

    async def abort_all(self):
        await self._post("/abort_request", {"abort_all": True})

    def payload(self, version):
        """The control record as SGLang's tensor-update route expects it, once per TP rank."""
        blob = base64.b64encode(pickle.dumps(control_payload(self.registry_url, version, self.member))).decode()
        return [blob] * self.tp_size

    async def update(self, version):
        await self._run([("/begin_weight_update", {}, True),
                         ("/update_weights_from_tensor", {"serialized_named_tensors": self.payload(version),
                                                          "load_format": LOADER, "flush_cache": True,
                                                          "weight_version": str(version)}, False),
                         ("/end_weight_update", {}, True)])
        self.version = version
