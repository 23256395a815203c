"""Deployment manifests and the PD membership sidecar on CPU: every kind
renders a valid List, GPU pods share the host IPC namespace and /dev/shm and
pin the node, the PD pods carry the ConnexConnector config and the
membership sidecar, options come from a config file, the environment and the
command line in that order, and the sidecar registers an instance while its
/health answers and deregisters it when it stops answering."""
import json
import threading

import pytest

from connex.deploy import k8s
from connex.pd import membership


def _items(*argv):
    out = k8s.generate(list(argv))
    assert out["kind"] == "List"
    return out["items"]


def _pod(items, name):
    d = next(i for i in items if i["kind"] == "Deployment" and i["metadata"]["name"] == name)
    return d["spec"]["template"]["spec"]


def test_every_kind_renders_deployments_with_services():
    for argv in (["router"], ["directory"], ["pd", "--model", "m"], ["ep", "--model", "m"],
                 ["proxy", "--endpoints", "http://a:1,http://b:2"]):
        items = _items(*argv)
        deps = {i["metadata"]["name"] for i in items if i["kind"] == "Deployment"}
        svcs = {i["metadata"]["name"] for i in items if i["kind"] == "Service"}
        assert deps and deps == svcs
        for i in items:
            assert i["metadata"]["namespace"] == "connex"
        json.dumps(items)


def test_pd_pods_share_ipc_and_carry_the_connector_and_sidecar():
    items = _items("pd", "--model", "llama", "--prefill", "2", "--decode", "3", "--node", "n1",
                   "--model-pvc", "models", "--namespace", "demo")
    names = [i["metadata"]["name"] for i in items if i["kind"] == "Deployment"]
    assert names == ["cx-prefill-0", "cx-prefill-1", "cx-decode-0", "cx-decode-1", "cx-decode-2", "cx-pd-router"]
    pod = _pod(items, "cx-decode-1")
    main, side = pod["containers"]
    assert pod["hostIPC"] is True and pod["nodeSelector"] == {"kubernetes.io/hostname": "n1"}
    assert {"name": "shm", "mountPath": "/dev/shm"} in main["volumeMounts"]
    assert main["resources"]["limits"] == {"nvidia.com/gpu": 1}
    kv = json.loads(main["command"][main["command"].index("--kv-transfer-config") + 1])
    assert kv["kv_connector"] == "ConnexConnector" and kv["kv_role"] == "kv_consumer"
    assert kv["kv_connector_module_path"] == "connex.adapters.vllm.pd_connector"
    assert main["command"][2] == "/models/llama"
    assert main["env"] == [{"name": "CONNEX_HOST_IP", "valueFrom": {"fieldRef": {"fieldPath": "status.podIP"}}}]
    assert side["command"][:3] == ["python", "-m", "connex.pd.membership"]
    assert side["command"][side["command"].index("--role") + 1] == "decode"
    assert side["command"][side["command"].index("--replica") + 1] == "1"
    router = _pod(items, "cx-pd-router")["containers"][0]["command"]
    assert "tcp://cx-front-router.demo.svc.cluster.local:15555" in router
    assert "hostIPC" not in _pod(items, "cx-pd-router")


def test_ep_pod_takes_all_gpus_with_the_worker_extension():
    pod = _pod(_items("ep", "--model", "q", "--gpus", "4"), "cx-ep")
    c = pod["containers"][0]
    assert c["resources"]["limits"] == {"nvidia.com/gpu": 4} and pod["hostIPC"] is True
    assert "connex.ep.vllm_ext.ConnexEPWorker" in c["command"] and "--enable-expert-parallel" in c["command"]
    assert {"name": "CONNEX_EP", "value": "1"} in c["env"]


def test_option_precedence_config_env_cli(tmp_path, monkeypatch):
    cfg = tmp_path / "c.json"
    cfg.write_text(json.dumps({"namespace": "from-file", "image": "file:1", "prefix": "p"}))
    monkeypatch.setenv("CONNEX_K8S_IMAGE", "env:2")
    items = _items("router", "--config", str(cfg), "--prefix", "cli")
    d = items[0]
    assert d["metadata"]["namespace"] == "from-file"
    assert d["spec"]["template"]["spec"]["containers"][0]["image"] == "env:2"
    assert d["metadata"]["name"] == "cli-front-router"


def test_missing_required_options_exit():
    with pytest.raises(SystemExit):
        k8s.generate(["pd"])
    with pytest.raises(SystemExit):
        k8s.generate(["proxy"])


def test_yaml_output(capsys):
    k8s.main(["router", "--yaml"])
    import yaml
    assert yaml.safe_load(capsys.readouterr().out)["kind"] == "List"


def test_sidecar_registers_while_healthy(monkeypatch):
    events = []

    class FakeMember:
        def __init__(self, fr, model, role, replica, url, **kw):
            self.args = (fr, model, role, replica, url)

        def start(self):
            events.append(("start",) + self.args)
            return True

        def stop(self):
            events.append(("stop", self.args[2]))
    monkeypatch.setattr(membership, "PDMember", FakeMember)
    health = iter([False, True, True, False, True])
    stop = threading.Event()

    def healthy(url):
        try:
            return next(health)
        except StopIteration:
            stop.set()
            return True
    membership.run_member("tcp://fr:1", "m", "prefill", 2, "http://p:8100", poll_s=0.0, stop=stop,
                          healthy=healthy)
    kinds = [e[0] for e in events]
    assert kinds == ["start", "stop", "start", "stop"]        # up, down, up again, deregistered at exit
    assert events[0] == ("start", "tcp://fr:1", "m", "prefill", 2, "http://p:8100")


def test_serve_and_pipeline_kinds_run_the_native_engine():
    items = _items("serve", "--model", "llama", "--replicas", "2", "--model-pvc", "models")
    assert [i["metadata"]["name"] for i in items if i["kind"] == "Deployment"] == ["cx-serve-0", "cx-serve-1"]
    c = _pod(items, "cx-serve-1")["containers"][0]
    assert c["command"][:3] == ["python", "-m", "connex_b200.serve"] and "/models/llama" in c["command"]
    assert c["readinessProbe"]["httpGet"]["path"] == "/health"
    items = _items("pipeline", "--model", "llama", "--num-stages", "3", "--stage-replicas", "2",
                   "--stage-starts", "10,20", "--namespace", "pp")
    deps = [i["metadata"]["name"] for i in items if i["kind"] == "Deployment"]
    assert deps == ["cx-directory", "cx-s0-r0", "cx-s1-r0", "cx-s1-r1", "cx-s2-r0", "cx-s2-r1"]
    s0 = _pod(items, "cx-s0-r0")["containers"][0]["command"]
    assert "--store-master" in s0 and s0[s0.index("--num-stages") + 1] == "3"
    assert s0[s0.index("--directory") + 1] == "cx-directory.pp.svc.cluster.local:15500"
    s2 = _pod(items, "cx-s2-r1")["containers"][0]["command"]
    assert s2[:3] == ["python", "-m", "connex_b200.serve.stage"]
    assert s2[s2.index("--stage") + 1] == "2" and s2[s2.index("--replica") + 1] == "1"
    assert s2[s2.index("--store") + 1] == "cx-s0-r0.pp.svc.cluster.local:29600"
    assert s2[s2.index("--stage-starts") + 1] == "10,20"
    d = _pod(items, "cx-directory")["containers"][0]["command"]
    assert d == ["connex-directory", "--bind", "0.0.0.0:15500", "--event-bind", "0.0.0.0:15501"]
    # every flag the manifests pass is one the CLIs accept
    import argparse
    from connex_b200.serve.__main__ import model_args
    ap = argparse.ArgumentParser()
    model_args(ap)
    ap.add_argument("--port")
    ap.add_argument("--stage")
    a = ap.parse_args(s0[3:])
    assert a.store_master and a.num_stages == 3
    a = ap.parse_args(s2[3:])
    assert a.replica == 1 and a.stage == "2"


def test_tensor_parallel_serve_replicas():
    c = _pod(_items("serve", "--model", "llama", "--tp", "4"), "cx-serve-0")["containers"][0]
    assert c["command"][:4] == ["torchrun", "--nproc-per-node", "4", "--master-addr"]
    assert c["command"][c["command"].index("--tp") + 1] == "4"
    assert c["resources"]["limits"] == {"nvidia.com/gpu": 4}
