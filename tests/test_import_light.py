"""``import connex`` and the control-plane / serving entry points stay light:
no torch, no vLLM, no native extension at import time."""
import subprocess
import sys

import pytest

PROBE = ("import sys, {mod}; heavy = [m for m in ('torch', 'vllm', 'connex_b200._C') if m in sys.modules]; "
         "print(','.join(heavy))")


@pytest.mark.parametrize("mod", ["connex", "connex.pp", "connex.front_router", "connex.directory_server",
                                 "connex.serving.proxy", "connex.serving.pd_router", "connex.agents",
                                 "connex.elastic", "connex.epc_client"])
def test_import_is_light(mod):
    r = subprocess.run([sys.executable, "-c", PROBE.format(mod=mod)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == "", f"{mod} imported {r.stdout.strip()}"


def test_lazy_names_resolve():
    import connex
    assert set(connex.__all__) <= set(dir(connex))
    assert connex.ElasticPeerSet.__name__ == "ElasticPeerSet"
    assert connex.PDRole.PREFILL == "prefill"
    assert connex.create_epc_client is connex.create_epc_client
    with pytest.raises(AttributeError):
        connex.no_such_name  # noqa: B018
