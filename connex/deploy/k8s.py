"""Kubernetes manifests for a Connex deployment on one NVLink/NVSwitch node
(the L7 deploy tool; the reference's is ``deploy/k8s/manifests.py``).

    python -m connex.deploy.k8s router --namespace demo --image REG/connex:TAG > router.json
    python -m connex.deploy.k8s pd --prefill 4 --decode 4 --model meta-llama/Meta-Llama-3-8B \\
        --node gpu-node-1 --model-pvc models > pd.json
    python -m connex.deploy.k8s ep --gpus 8 --model Qwen/Qwen3-30B-A3B --node gpu-node-1 > ep.json
    python -m connex.deploy.k8s proxy --endpoints http://a:8000,http://b:8000 > proxy.json
    python -m connex.deploy.k8s serve --replicas 4 --model Meta-Llama-3-8B --model-pvc models > serve.json
    python -m connex.deploy.k8s pipeline --num-stages 2 --stage-replicas 2 --model Meta-Llama-3-8B \
        --model-pvc models --node gpu-node-1 > pipeline.json
    kubectl apply -f router.json -f pd.json

Output is a ``v1/List`` in JSON (``--yaml`` for YAML).  Options come from the
command line, a ``--config`` JSON object (keys = long option names with ``_``)
or ``CONNEX_K8S_<OPTION>`` environment variables, in increasing precedence
from config file to environment to command line.

Why the GPU pods share one node, the host IPC namespace and ``/dev/shm``:
the data paths of this framework move KV blocks, expert weights and weight
versions between GPUs by CUDA IPC handles of peer memory over NVLink, and the
same-host region records live in ``/dev/shm``; both need the pods of one box
to see each other's IPC objects.  Each GPU pod asks for one
``nvidia.com/gpu`` (``--gpu-resource``); the device plugin picks the GPU.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from typing import Dict, List, Optional

DEFAULTS = {
    "namespace": "connex",
    "image": "connex:latest",
    "prefix": "cx",
    "node": "",
    "model": "",
    "model_pvc": "",
    "model_host_path": "",
    "gpu_resource": "nvidia.com/gpu",
    "prefill": 1,
    "decode": 1,
    "gpus": 8,
    "router_port": 15555,
    "events_port": 15560,
    "pd_router_port": 8000,
    "serve_port": 8100,
    "proxy_port": 5199,
    "ctrl_port": 17100,
    "replicas": 1,
    "tp": 1,
    "num_stages": 2,
    "stage_replicas": 1,
    "stage_starts": "",
    "directory_port": 15500,
    "store_port": 29600,
    "max_ctx": 4096,
    "max_batch": 64,
    "endpoints": "",
}
KINDS = ("router", "directory", "pd", "ep", "proxy", "serve", "pipeline")


POD_IP = object()     # env value: the pod's own IP from the downward API


def _env(d: Dict[str, object]) -> List[dict]:
    return [{"name": k, "valueFrom": {"fieldRef": {"fieldPath": "status.podIP"}}} if v is POD_IP
            else {"name": k, "value": str(v)} for k, v in d.items() if v not in (None, "")]


def _labels(c, name: str) -> dict:
    return {"app.kubernetes.io/part-of": c["prefix"], "app.kubernetes.io/name": name}


def _service(c, name: str, ports: Dict[str, int]) -> dict:
    return {"apiVersion": "v1", "kind": "Service",
            "metadata": {"name": name, "namespace": c["namespace"], "labels": _labels(c, name)},
            "spec": {"selector": _labels(c, name),
                     "ports": [{"name": n, "port": p, "targetPort": p} for n, p in ports.items()]}}


def _deployment(c, name: str, command: List[str], env: dict, ports: Dict[str, int], gpus: int = 0,
                sidecars: Optional[List[dict]] = None) -> dict:
    container = {"name": name, "image": c["image"], "command": command, "env": _env(env),
                 "ports": [{"name": n, "containerPort": p} for n, p in ports.items()]}
    pod: dict = {"containers": [container] + list(sidecars or [])}
    if gpus:
        container["resources"] = {"limits": {c["gpu_resource"]: gpus}}
        # CUDA IPC handles and /dev/shm region records are shared by the GPU pods of the node
        pod["hostIPC"] = True
        pod["volumes"] = [{"name": "shm", "hostPath": {"path": "/dev/shm", "type": "Directory"}}]
        container["volumeMounts"] = [{"name": "shm", "mountPath": "/dev/shm"}]
        if c["model_pvc"]:
            pod["volumes"].append({"name": "model", "persistentVolumeClaim": {"claimName": c["model_pvc"],
                                                                             "readOnly": True}})
            container["volumeMounts"].append({"name": "model", "mountPath": "/models", "readOnly": True})
        elif c["model_host_path"]:
            pod["volumes"].append({"name": "model", "hostPath": {"path": c["model_host_path"], "type": "Directory"}})
            container["volumeMounts"].append({"name": "model", "mountPath": "/models", "readOnly": True})
    if c["node"]:
        pod["nodeSelector"] = {"kubernetes.io/hostname": c["node"]}
    return {"apiVersion": "apps/v1", "kind": "Deployment",
            "metadata": {"name": name, "namespace": c["namespace"], "labels": _labels(c, name)},
            "spec": {"replicas": 1, "selector": {"matchLabels": _labels(c, name)},
                     "template": {"metadata": {"labels": _labels(c, name)}, "spec": pod}}}


def _router_url(c) -> str:
    return f"tcp://{c['prefix']}-front-router.{c['namespace']}.svc.cluster.local:{c['router_port']}"


def _model_arg(c) -> str:
    if not c["model"]:
        raise SystemExit("--model is required")
    return f"/models/{c['model']}" if (c["model_pvc"] or c["model_host_path"]) else c["model"]


def router(c) -> List[dict]:
    name = f"{c['prefix']}-front-router"
    ports = {"api": c["router_port"], "events": c["events_port"]}
    cmd = ["connex-front-router", "--api-address", f"tcp://*:{c['router_port']}",
           "--event-address", f"tcp://*:{c['events_port']}"]
    return [_deployment(c, name, cmd, {}, ports), _service(c, name, ports)]


def directory(c) -> List[dict]:
    name = f"{c['prefix']}-directory"
    port = c["directory_port"]
    ports = {"dir": port, "events": port + 1}
    cmd = ["connex-directory", "--bind", f"0.0.0.0:{port}", "--event-bind", f"0.0.0.0:{port + 1}"]
    return [_deployment(c, name, cmd, {}, ports), _service(c, name, ports)]


def pd(c) -> List[dict]:
    """Prefill and decode vLLM instances with the ConnexConnector (KV over
    NVLink peer memory), registered in the front-router PD pools, and the PD
    router in front of them."""
    items: List[dict] = []
    model = _model_arg(c)
    events = f"tcp://{c['prefix']}-front-router.{c['namespace']}.svc.cluster.local:{c['events_port']}"
    for role, n in (("prefill", c["prefill"]), ("decode", c["decode"])):
        for r in range(int(n)):
            name = f"{c['prefix']}-{role}-{r}"
            url = f"http://{name}.{c['namespace']}.svc.cluster.local:{c['serve_port']}"
            kv = {"kv_connector": "ConnexConnector", "kv_connector_module_path": "connex.adapters.vllm.pd_connector",
                  "kv_role": "kv_producer" if role == "prefill" else "kv_consumer",
                  "kv_connector_extra_config": {"backend": "nvlink", "ctrl_port": c["ctrl_port"]}}
            cmd = ["vllm", "serve", model, "--port", str(c["serve_port"]), "--kv-transfer-config", json.dumps(kv)]
            # the sidecar keeps the instance in the front-router PD pool while /health answers
            member = {"name": "pd-member", "image": c["image"],
                      "command": ["python", "-m", "connex.pd.membership", "--front-router", _router_url(c),
                                  "--model", c["model"], "--role", role, "--replica", str(r), "--url", url]}
            items += [_deployment(c, name, cmd, {"CONNEX_HOST_IP": POD_IP},
                                  {"http": c["serve_port"], "kv-ctrl": c["ctrl_port"]},
                                  gpus=1, sidecars=[member]),
                      _service(c, name, {"http": c["serve_port"]})]
    name = f"{c['prefix']}-pd-router"
    cmd = ["connex-pd-router", "--port", str(c["pd_router_port"]), "--front-router", _router_url(c),
           "--front-router-events", events, "--model", c["model"]]
    items += [_deployment(c, name, cmd, {}, {"http": c["pd_router_port"]}),
              _service(c, name, {"http": c["pd_router_port"]})]
    return items


def ep(c) -> List[dict]:
    """One vLLM server spanning ``--gpus`` GPUs with expert parallelism and
    the Connex EP worker extension (placement owned by an EPController)."""
    name = f"{c['prefix']}-ep"
    cmd = ["vllm", "serve", _model_arg(c), "--port", str(c["serve_port"]), "--enable-expert-parallel",
           "--data-parallel-size", str(c["gpus"]), "--enable-eplb",
           "--worker-extension-cls", "connex.ep.vllm_ext.ConnexEPWorker"]
    env = {"CONNEX_EP": 1, "VLLM_SERVER_DEV_MODE": 1}
    return [_deployment(c, name, cmd, env, {"http": c["serve_port"]}, gpus=int(c["gpus"])),
            _service(c, name, {"http": c["serve_port"]})]


def proxy(c) -> List[dict]:
    if not c["endpoints"]:
        raise SystemExit("--endpoints is required (comma-separated replica URLs)")
    name = f"{c['prefix']}-proxy"
    cmd = ["connex-proxy", "--port", str(c["proxy_port"]), "--endpoints", c["endpoints"]]
    return [_deployment(c, name, cmd, {}, {"http": c["proxy_port"]}), _service(c, name, {"http": c["proxy_port"]})]


def _engine_args(c) -> List[str]:
    return ["--checkpoint", _model_arg(c), "--model-name", c["model"], "--max-ctx", str(c["max_ctx"]),
            "--max-batch", str(c["max_batch"]), "--device", "cuda:0"]


def _ready(container: dict, port: int) -> None:
    container["readinessProbe"] = {"httpGet": {"path": "/health", "port": port}, "periodSeconds": 5,
                                   "failureThreshold": 3}


def serve(c) -> List[dict]:
    """``--replicas`` servers of this framework's own engine (``python -m
    connex_b200.serve``; ``--tp N`` GPUs each, tensor-parallel under
    torchrun), each behind its Service; put the ``proxy`` kind in front of
    them for retries and stream resume."""
    items: List[dict] = []
    tp = int(c["tp"])
    for r in range(int(c["replicas"])):
        name = f"{c['prefix']}-serve-{r}"
        if tp > 1:          # one process per GPU; rank 0 serves HTTP
            cmd = ["torchrun", "--nproc-per-node", str(tp), "--master-addr", "127.0.0.1", "-m", "connex_b200.serve",
                   "--tp", str(tp), "--port", str(c["serve_port"])] + _engine_args(c)
        else:
            cmd = ["python", "-m", "connex_b200.serve", "--port", str(c["serve_port"])] + _engine_args(c)
        d = _deployment(c, name, cmd, {}, {"http": c["serve_port"]}, gpus=tp)
        _ready(d["spec"]["template"]["spec"]["containers"][0], c["serve_port"])
        items += [d, _service(c, name, {"http": c["serve_port"]})]
    return items


def pipeline(c) -> List[dict]:
    """An elastic serving pipeline of this framework's engine: a directory,
    stage 0 (OpenAI API; hosts the pair-link rendezvous store) and
    ``--stage-replicas`` replicas of every later stage, one GPU each.  Stage
    endpoints register their pod address in the directory; stage 0 fails
    over to another replica of stage 1.. when one dies."""
    items = directory(c)
    ns = c["namespace"]
    dir_addr = f"{c['prefix']}-directory.{ns}.svc.cluster.local:{c['directory_port']}"
    s0 = f"{c['prefix']}-s0-r0"
    store = f"{s0}.{ns}.svc.cluster.local:{c['store_port']}"
    common = _engine_args(c) + ["--num-stages", str(c["num_stages"]), "--directory", dir_addr, "--store", store]
    if c["stage_starts"]:
        common += ["--stage-starts", c["stage_starts"]]
    env = {"CONNEX_HOST_IP": POD_IP}
    cmd = ["python", "-m", "connex_b200.serve", "--port", str(c["serve_port"]), "--store-master"] + common
    ports = {"http": c["serve_port"], "store": c["store_port"]}
    d = _deployment(c, s0, cmd, env, ports, gpus=1)
    _ready(d["spec"]["template"]["spec"]["containers"][0], c["serve_port"])
    items += [d, _service(c, s0, ports)]
    for k in range(1, int(c["num_stages"])):
        for r in range(int(c["stage_replicas"])):
            name = f"{c['prefix']}-s{k}-r{r}"
            cmd = ["python", "-m", "connex_b200.serve.stage", "--stage", str(k), "--replica", str(r)] + common
            items.append(_deployment(c, name, cmd, env, {}, gpus=1))
    return items


def _options(argv: Optional[List[str]]) -> dict:
    pre = argparse.ArgumentParser(add_help=False)
    pre.add_argument("--config")
    known, _ = pre.parse_known_args(argv)
    opts = dict(DEFAULTS)
    if known.config:
        with open(known.config) as f:
            opts.update(json.load(f))
    for k in DEFAULTS:
        v = os.environ.get(f"CONNEX_K8S_{k.upper()}")
        if v is not None:
            opts[k] = type(DEFAULTS[k])(v)
    p = argparse.ArgumentParser(description="Kubernetes manifests for a Connex deployment")
    p.add_argument("what", choices=KINDS)
    p.add_argument("--config")
    p.add_argument("--yaml", action="store_true")
    for k, v in DEFAULTS.items():
        p.add_argument("--" + k.replace("_", "-"), dest=k, type=type(v), default=opts[k])
    a = p.parse_args(argv)
    return vars(a)


def generate(argv: Optional[List[str]] = None) -> dict:
    c = _options(argv)
    items = {"router": router, "directory": directory, "pd": pd, "ep": ep, "proxy": proxy, "serve": serve,
             "pipeline": pipeline}[c["what"]](c)
    return {"apiVersion": "v1", "kind": "List", "items": items}


def main(argv: Optional[List[str]] = None) -> int:
    out = generate(argv)
    if "--yaml" in (argv if argv is not None else sys.argv[1:]):
        import yaml
        print(yaml.safe_dump(out, sort_keys=False))
    else:
        print(json.dumps(out, indent=1))
    return 0


if __name__ == "__main__":
    sys.exit(main())
