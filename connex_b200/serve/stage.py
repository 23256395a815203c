"""``python -m connex_b200.serve.stage`` -- a downstream replica of a
serving pipeline: layers ``[l0, l1)`` of the model on this GPU, answering
the step protocol of stage 0 (``python -m connex_b200.serve --num-stages
S``) through its endpoint.  Start several replicas of a stage (``--replica
R``) for failover: stage 0 moves to another one when this one dies and
re-prefills the rows whose KV it lacks.

    python -m connex_b200.serve.stage --checkpoint CK --num-stages 2 --stage 1 --replica 0 \\
        --directory 127.0.0.1:15500 --store 127.0.0.1:29600
"""
from __future__ import annotations

import argparse
import logging
import signal
import threading

from connex_b200.serve.__main__ import kv_blocks, llama_config, model_args

log = logging.getLogger("connex_b200.serve.stage")


def run_stage(a, stop: threading.Event) -> dict:
    import torch

    from connex.pp.link import StageWorker
    if a.rule:                 # CPU stand-in stage (no GPU): ids as activations, ids as KV
        from connex_b200.serve import pipeline
        from connex_b200.serve.engine import RuleStageRuntime
        rt = RuleStageRuntime(False, a.stage == a.num_stages - 1, 1000, a.rule_delay_ms / 1e3)
        ep, client = pipeline.join(a.model_name or "connex-b200", a.stage, a.num_stages, a.replica, "cpu",
                                   a.directory, "inline", None, False, a.advertise_host, a.recv_timeout_s)
        return _serve_loop(ep, client, StageWorker(ep, rt, rt.compute), stop, a, (a.stage, a.stage + 1))
    from connex_b200.models.hf import load_llama
    from connex_b200.runtime.pp import StageRuntime
    from connex_b200.serve import pipeline
    cfg = llama_config(a)
    dev = torch.device(a.device)
    torch.cuda.set_device(dev)
    l0, l1 = pipeline.split_layers(cfg.layers, a.num_stages, a.stage_starts)[a.stage]
    weights = load_llama(a.checkpoint, dev, layers=(l0, l1), cfg=cfg) if a.checkpoint else None
    rt = StageRuntime(cfg, l0, l1, dev, num_blocks=kv_blocks(a, cfg, l0, l1), max_tokens=a.max_step_tokens,
                      max_batch=a.max_batch, max_ctx=a.max_ctx, seed=a.seed, weights=weights)
    if not a.no_graphs:
        rt.enable_decode_graphs()
    ep, client = pipeline.join(a.model_name or "connex-b200", a.stage, a.num_stages, a.replica, dev, a.directory,
                               a.data, a.store, a.store_master, a.advertise_host, a.recv_timeout_s)
    return _serve_loop(ep, client, StageWorker(ep, rt, rt.compute), stop, a, (l0, l1))


def _serve_loop(ep, client, worker, stop: threading.Event, a, layers) -> dict:
    from connex_b200.serve import pipeline
    log.info("stage %d replica %d: layers [%d, %d) serving at %s", a.stage, a.replica, layers[0], layers[1],
             ep.address)
    try:
        while not stop.is_set():
            td, ctx = ep.recv_forward(timeout_s=0.2)
            if td is not None:
                worker.serve(td, ctx)
    finally:
        pipeline.leave(ep, client)
    return dict(worker.stats)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="downstream stage of a serving pipeline")
    model_args(ap)
    ap.add_argument("--stage", type=int, required=True)
    ap.add_argument("--rule", action="store_true", help="CPU stand-in stage (with a --rule stage 0)")
    ap.add_argument("--rule-delay-ms", type=float, default=0.0, help="stand-in stage: sleep per step")
    ap.add_argument("--log-level", default="INFO")
    a = ap.parse_args(argv)
    if not 0 < a.stage < a.num_stages or not a.directory:
        raise SystemExit("--stage must lie in [1, --num-stages) and --directory is required")
    logging.basicConfig(level=getattr(logging, a.log_level), format="%(asctime)s [%(levelname)s] %(name)s: %(message)s")
    stop = threading.Event()
    signal.signal(signal.SIGTERM, lambda *_: stop.set())
    signal.signal(signal.SIGINT, lambda *_: stop.set())
    run_stage(a, stop)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
