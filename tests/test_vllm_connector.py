"""``ConnexConnector`` against vLLM's connector base class on CPU: the
scheduler-side protocol (hold on the prefill, external tokens + async load
on the decode, release at the end) and the worker-side pull over the
loopback data plane, block for block."""
from types import SimpleNamespace

import pytest
import torch

pytest.importorskip("vllm.distributed.kv_transfer.kv_connector.v1.base")


def _cfg(role, port):
    tc = SimpleNamespace(kv_role=role, kv_port=port,
                         kv_connector_extra_config={"backend": "loopback", "ctrl_port": port, "host": "127.0.0.1",
                                                    "bind_ip": "127.0.0.1"})
    return SimpleNamespace(kv_transfer_config=tc, cache_config=SimpleNamespace(block_size=16))


class Blocks:
    def __init__(self, ids):
        self.ids = ids

    def get_block_ids(self):
        return (self.ids,)


def _req(rid, n, params):
    return SimpleNamespace(request_id=rid, prompt_token_ids=list(range(n)), kv_transfer_params=params)


def test_connector_hold_pull_release_roundtrip():
    import socket
    import time
    from vllm.distributed.kv_transfer.kv_connector.v1.base import KVConnectorRole
    from connex.adapters.vllm.pd_connector import ConnexConnector
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    NB = 12
    kvc = SimpleNamespace(num_blocks=NB)
    pre_caches = {f"l{i}": torch.randn(2, NB, 16, 2, 64) for i in range(2)}
    dec_caches = {f"l{i}": torch.zeros(2, NB, 16, 2, 64) for i in range(2)}
    p_sched = ConnexConnector(_cfg("kv_producer", port), KVConnectorRole.SCHEDULER, kvc)
    p_work = ConnexConnector(_cfg("kv_producer", port), KVConnectorRole.WORKER, kvc)
    d_sched = ConnexConnector(_cfg("kv_consumer", port + 50), KVConnectorRole.SCHEDULER, kvc)
    d_work = ConnexConnector(_cfg("kv_consumer", port + 50), KVConnectorRole.WORKER, kvc)
    p_work.register_kv_caches(pre_caches)
    d_work.register_kv_caches(dec_caches)
    try:
        # prefill finishes: blocks kept, params returned, worker holds them
        delay, params = p_sched.request_finished(_req("r1", 40, {"do_remote_decode": True, "transfer_id": "T1"}),
                                                 [3, 5, 7])
        assert delay and params["transfer_id"] == "T1" and params["remote_num_tokens"] == 40
        p_work.bind_connector_metadata(p_sched.build_connector_meta(None))
        p_work.start_load_kv(None)
        # decode: the prompt is external, loaded asynchronously into its own blocks
        r2 = _req("r2", 40, params)
        assert d_sched.get_num_new_matched_tokens(r2, 0) == (40, True)
        d_sched.update_state_after_alloc(r2, Blocks([1, 2, 9]), 40)
        assert d_sched.get_num_new_matched_tokens(r2, 40) == (0, False)
        d_work.bind_connector_metadata(d_sched.build_connector_meta(None))
        d_work.start_load_kv(None)
        deadline = time.time() + 10
        recv = set()
        while time.time() < deadline and "r2" not in recv:
            _, got = d_work.get_finished(set())
            recv |= got or set()
            time.sleep(0.02)
        assert "r2" in recv and not d_work.get_block_ids_with_load_errors()
        for name in pre_caches:
            assert torch.equal(dec_caches[name][:, [1, 2, 9]], pre_caches[name][:, [3, 5, 7]])
        # the decode finishes: release -> the prefill frees its blocks
        assert d_sched.request_finished(r2, [1, 2, 9]) == (False, None)
        d_work.bind_connector_metadata(d_sched.build_connector_meta(None))
        d_work.start_load_kv(None)
        sent = set()
        deadline = time.time() + 10
        while time.time() < deadline and "r1" not in sent:
            got, _ = p_work.get_finished(set())
            sent |= got or set()
            time.sleep(0.02)
        assert "r1" in sent
    finally:
        p_work.shutdown()
        d_work.shutdown()


def test_plugin_registers_connector():
    from vllm.distributed.kv_transfer.kv_connector.factory import KVConnectorFactory
    from connex.adapters.vllm.plugin import register
    register()
    register()
    assert "ConnexConnector" in KVConnectorFactory._registry
