"""``python -m connex_b200.serve`` -- OpenAI-compatible server over this
framework's Llama runtime.

One GPU, all layers::

    python -m connex_b200.serve --checkpoint /models/Meta-Llama-3-8B --port 8100

Stage 0 of a two-stage pipeline (downstream replicas run
``python -m connex_b200.serve.stage``; both register with a directory)::

    connex-directory --bind 0.0.0.0:15500 &
    python -m connex_b200.serve --checkpoint CK --num-stages 2 --directory 127.0.0.1:15500 \\
        --store 127.0.0.1:29600 --store-master --port 8100

Without ``--checkpoint`` the weights are random with the geometry of
``--config`` (``llama3-8b`` or ``tiny``), and prompts / outputs use the word
codec (``t<id>``).  ``--rule`` serves the deterministic CPU stand-in model
(no GPU), for wiring checks.
"""
from __future__ import annotations

import argparse
import asyncio
import logging
import os
import signal

log = logging.getLogger("connex_b200.serve")


def model_args(ap: argparse.ArgumentParser) -> None:
    ap.add_argument("--checkpoint", default=None, help="HF Llama checkpoint directory (config.json + safetensors)")
    ap.add_argument("--config", default="llama3-8b", choices=["llama3-8b", "llama3.1-8b", "tiny"],
                    help="geometry of random weights when no checkpoint is given (llama3.1-8b: 128k positions, "
                         "Llama 3.1 RoPE scaling)")
    ap.add_argument("--layers", type=int, default=None, help="override the layer count of --config")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--device", default="cuda:0")
    ap.add_argument("--num-blocks", type=int, default=0, help="KV blocks (0: from --kv-fraction of free memory)")
    ap.add_argument("--kv-fraction", type=float, default=0.8)
    ap.add_argument("--max-batch", type=int, default=64)
    ap.add_argument("--max-ctx", type=int, default=4096)
    ap.add_argument("--max-step-tokens", type=int, default=8192)
    ap.add_argument("--model-name", default=None)
    ap.add_argument("--num-stages", type=int, default=1)
    ap.add_argument("--stage-starts", default=None, help="first layer of stages 1.. (even split by default)")
    ap.add_argument("--directory", default=None, help="HOST:PORT of the directory (connex-directory --bind)")
    ap.add_argument("--data", default="link", choices=["link", "inline"])
    ap.add_argument("--store", default=None, help="HOST:PORT of the pair-link rendezvous store")
    ap.add_argument("--store-master", action="store_true", help="host the rendezvous store in this process")
    ap.add_argument("--replica", type=int, default=0)
    ap.add_argument("--advertise-host", default=os.getenv("CONNEX_HOST_IP", "127.0.0.1"),
                    help="address the pipeline endpoint binds and advertises")
    ap.add_argument("--recv-timeout-s", type=float, default=30.0)
    ap.add_argument("--step-timeout-s", type=float, default=60.0,
                    help="stage 0: the step watchdog's fixed timeout (until enough steps were measured)")
    ap.add_argument("--no-graphs", action="store_true", help="launch decode steps eagerly (no CUDA graphs)")
    ap.add_argument("--tp", type=int, default=1,
                    help="tensor-parallel ranks (launch with torchrun --nproc-per-node TP; rank 0 serves HTTP)")


def llama_config(a):
    from connex_b200.models.llama import LlamaConfig
    if a.checkpoint:
        from connex_b200.models.hf import config_from_hf
        cfg = config_from_hf(a.checkpoint)
    else:
        cfg = {"tiny": LlamaConfig.tiny, "llama3.1-8b": LlamaConfig.llama31_8b}.get(a.config, LlamaConfig.llama3_8b)()
    if a.layers:
        cfg = LlamaConfig(**{**cfg.__dict__, "layers": a.layers})
    if a.max_ctx > cfg.max_pos:
        raise SystemExit(f"--max-ctx {a.max_ctx} exceeds the model's positions ({cfg.max_pos})")
    return cfg


def kv_blocks(a, cfg, l0: int, l1: int) -> int:
    """``--num-blocks``, or the blocks of layers [l0, l1) that fit in
    ``--kv-fraction`` of the device memory free after the weights (an
    estimate of the weights' bytes is subtracted before they are loaded)."""
    if a.num_blocks:
        return a.num_blocks
    import torch
    free, _ = torch.cuda.mem_get_info(torch.device(a.device))
    n_layers = l1 - l0
    per_layer = cfg.qkv_dim * cfg.hidden + cfg.hidden * cfg.heads * cfg.head_dim + 3 * cfg.ffn * cfg.hidden
    weights = 2 * (n_layers * per_layer + 2 * cfg.vocab_size * cfg.hidden)
    block = 2 * n_layers * cfg.kv_heads * cfg.block_size * cfg.head_dim * 2
    scratch = 2 << 30                       # activations, workspaces, allocator slack
    return max(64, int((free - weights - scratch) * a.kv_fraction) // block)


def build_stepper(a):
    from connex_b200.serve.engine import ModelStepper, PipelineStepper, RuleStepper
    if getattr(a, "rule", False) and a.num_stages > 1:
        return _rule_pipeline(a)
    if getattr(a, "rule", False):
        return RuleStepper(vocab_size=1000, max_batch=a.max_batch, max_ctx=a.max_ctx), None
    import torch
    cfg = llama_config(a)
    if getattr(a, "tp", 1) > 1:
        return _tp_stepper(a, cfg)
    dev = torch.device(a.device)
    torch.cuda.set_device(dev)
    if a.num_stages == 1:
        n = kv_blocks(a, cfg, 0, cfg.layers)
        return ModelStepper(cfg, dev, n, a.max_batch, a.max_ctx, a.max_step_tokens, a.checkpoint, a.seed,
                            graphs=not a.no_graphs), None
    from connex_b200.serve import pipeline
    ranges = pipeline.split_layers(cfg.layers, a.num_stages, a.stage_starts)
    if not a.directory:
        raise SystemExit("--num-stages > 1 needs --directory")
    n = kv_blocks(a, cfg, *ranges[0])
    ep, client = pipeline.join(a.model_name or "connex-b200", 0, a.num_stages, a.replica, dev, a.directory, a.data,
                               a.store, a.store_master, a.advertise_host, a.recv_timeout_s)
    st = PipelineStepper(cfg, ranges[0][1], dev, ep, n, a.max_batch, a.max_ctx, a.max_step_tokens, a.checkpoint,
                         a.seed, a.recv_timeout_s, graphs=not a.no_graphs)
    ep.warm_stage(1)
    ep.auto_warm = True
    ep.watchdog = pipeline.watchdog(ep, st.link, client, step_timeout=a.step_timeout_s)
    return st, (ep, client)


def _rule_pipeline(a):
    """Stage 0 of a pipeline of CPU stand-in stages (``--rule``: every stage
    runs :class:`RuleStageRuntime`; ``--data inline``), to check the CLIs,
    the directory and failover without a GPU."""
    from connex_b200.models.llama import LlamaConfig
    from connex_b200.serve import pipeline
    from connex_b200.serve.engine import PipelineStepper, RuleStageRuntime
    if not a.directory:
        raise SystemExit("--num-stages > 1 needs --directory")
    cfg = LlamaConfig(vocab_size=1000)
    ep, client = pipeline.join(a.model_name or "connex-b200", 0, a.num_stages, a.replica, "cpu", a.directory, "inline",
                               None, False, a.advertise_host, a.recv_timeout_s)
    st = PipelineStepper(cfg, 1, "cpu", ep, 1 << 20, a.max_batch, a.max_ctx, a.max_step_tokens,
                         recv_timeout_s=a.recv_timeout_s, rt=RuleStageRuntime(True, False, 1000))
    ep.warm_stage(1)
    ep.auto_warm = True
    ep.watchdog = pipeline.watchdog(ep, st.link, client, step_timeout=a.step_timeout_s)
    return st, (ep, client)


def _tp_stepper(a, cfg):
    """Tensor-parallel serving: one process per GPU (torchrun); rank 0 gets a
    TPStepper, the other ranks follow rank 0's steps here and return None.
    Decode CUDA graphs stay off under TP (the all-reduces run eagerly)."""
    import datetime

    import torch
    import torch.distributed as dist

    from connex_b200.parallel.tp import TPGroup
    from connex_b200.serve.engine import ModelStepper, TPStepper, tp_follow
    if a.num_stages != 1:
        raise SystemExit("--tp with --num-stages > 1 is not supported")
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    if world != a.tp:
        raise SystemExit(f"--tp {a.tp} but WORLD_SIZE {world}")
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    cpu = dist.new_group(backend="gloo")
    from connex_b200.parallel.tp import tp_config
    blocks = kv_blocks(argparse.Namespace(**{**vars(a), "device": str(dev)}), tp_config(cfg, world), 0, cfg.layers)
    t = torch.tensor([blocks], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MIN)              # every rank sizes its KV cache alike
    inner = ModelStepper(cfg, dev, int(t.item()), a.max_batch, a.max_ctx, a.max_step_tokens, a.checkpoint,
                         a.seed, graphs=False, tp=TPGroup(rank, world))
    if rank == 0:
        return TPStepper(inner, cpu), ("tp", cpu)
    log.info("TP rank %d of %d following rank 0", rank, world)
    n = tp_follow(inner, cpu)
    log.info("TP rank %d: rank 0 stopped after %d steps", rank, n)
    dist.destroy_process_group()
    return None, None


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="OpenAI-compatible server over the sm_100a Llama runtime")
    model_args(ap)
    ap.add_argument("--host", default="0.0.0.0")
    ap.add_argument("--port", type=int, default=8100)
    ap.add_argument("--tokenizer", default=None, help="HF tokenizer directory (default: the checkpoint's, if any)")
    ap.add_argument("--rule", action="store_true", help="serve the deterministic CPU stand-in model (with "
                    "--num-stages: stage 0 of a pipeline of stand-in stages)")
    ap.add_argument("--log-level", default="INFO")
    a = ap.parse_args(argv)
    logging.basicConfig(level=getattr(logging, a.log_level), format="%(asctime)s [%(levelname)s] %(name)s: %(message)s")
    from connex_b200.serve.api import HFCodec, Server, serve
    from connex_b200.serve.engine import GenerationEngine
    stepper, pp = build_stepper(a)
    if stepper is None:                 # a tensor-parallel follower rank: done
        return 0
    tok_dir = a.tokenizer or (a.checkpoint if a.checkpoint and os.path.exists(
        os.path.join(a.checkpoint, "tokenizer_config.json")) else None)
    codec = HFCodec(tok_dir) if tok_dir else None
    engine = GenerationEngine(stepper).start()
    server = Server(engine, a.model_name or (os.path.basename(a.checkpoint.rstrip("/")) if a.checkpoint
                                             else "connex-b200"), codec)

    async def run():
        runner, port = await serve(server, a.host, a.port)
        log.info("serving %s on %s:%d (%s)", server.model, a.host, port,
                 f"{a.num_stages} stages" if a.num_stages > 1 else "one GPU" if not a.rule else "rule model")
        stop = asyncio.Event()
        loop = asyncio.get_running_loop()
        for sig in (signal.SIGINT, signal.SIGTERM):
            loop.add_signal_handler(sig, stop.set)
        await stop.wait()
        await runner.cleanup()
    try:
        asyncio.run(run())
    finally:
        engine.stop()
        if pp is not None and pp[0] == "tp":
            stepper.close()             # releases the follower ranks
            import torch.distributed as dist
            dist.destroy_process_group()
        elif pp is not None:
            from connex_b200.serve import pipeline
            pipeline.leave(*pp)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
