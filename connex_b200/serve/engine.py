"""Continuous-batching generation over this framework's Llama runtime.

:class:`GenerationEngine` owns one thread that drives a *stepper* (the
model): each iteration admits waiting requests that fit (batch slots, KV
blocks reserved for prompt + ``max_tokens``), then runs one step and hands
each new token to the request's callback.  A request ends at
``max_tokens``, at a stop id, or when it is cancelled (client gone); its KV
blocks are released at once.

Chunked prefill (steppers with ``supports_mixed``): every step is one
*mixed* batch -- a decode row (one token) for each request that is
generating, plus prefill chunks of the prompts still being read, up to the
step's token budget (``max_step_tokens``) in admission order.  A prompt
longer than the budget is read over several steps while the others keep
decoding (a 30k-token prompt no longer stalls every stream for its whole
prefill); its first token comes from the step with its last chunk.  Every
GEMM of a step runs once over all its rows.  Steppers without mixed steps
get a prefill step for the admitted prompts (whole, within the budget) and a
decode step per iteration.

Steppers:

* :class:`ModelStepper` -- one GPU, all layers (:class:`StageRuntime` over
  ``[0, L)``), weights random or from an HF checkpoint;
* :class:`PipelineStepper` -- stage 0 of an elastic pipeline: its layers
  locally, the rest through a :class:`connex.pp.link.Stage0Link`; rows whose
  KV a failed-over downstream replica does not hold are prefilled again with
  prompt + generated tokens, which yields the same next token;
* :class:`RuleStepper` -- a deterministic CPU stand-in (next id = a function
  of the last two ids), for tests of the scheduler and the HTTP layer.

Reference behaviour served this way: the OpenAI API of a vLLM stage-0
instance behind the proxy / PD router (``connex/serving/proxy.py``,
``connex/adapters/vllm/pp``); the engine itself is this framework's own.
"""
from __future__ import annotations

import collections
import itertools
import logging
import threading
import time
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Sequence

from connex.pp.handover import CX_CTX, REQUEST_IDS

log = logging.getLogger("connex_b200.serve")


class Stepper:
    """The model behind a :class:`GenerationEngine`.

    ``prefill(rids, seqs)`` computes every token of each sequence (KV written
    for all of them) and returns the greedy next id per sequence;
    ``decode(rids, seqs)`` appends the last id of each sequence (whose
    earlier ids are already in the KV cache) and returns the next ids;
    ``release(rids)`` frees their KV."""

    max_batch: int = 64
    max_ctx: int = 4096
    max_step_tokens: int = 8192
    num_blocks: int = 1 << 30
    block_size: int = 16
    vocab_size: int = 0
    supports_mixed: bool = False

    def prefill(self, rids: List[str], seqs: List[List[int]]) -> List[int]:
        raise NotImplementedError

    def mixed(self, rids: List[str], seqs: List[List[int]], ctx: List[int], n_new: List[int]) -> List[int]:
        """One step over rows that each add ``seq[ctx:ctx + n_new]`` to a
        sequence whose first ``ctx`` ids are already in the KV cache (decode
        rows and prefill chunks together); returns each row's greedy next id
        (the one after ``seq[ctx + n_new - 1]``)."""
        raise NotImplementedError

    def decode(self, rids: List[str], seqs: List[List[int]]) -> List[int]:
        raise NotImplementedError

    def release(self, rids: List[str]) -> None:
        pass

    def close(self) -> None:
        pass


class RuleStepper(Stepper):
    """Greedy stand-in on the CPU: the next id is
    :func:`connex.serving.fake_backend.next_token` of the last two ids (the
    fake HTTP backend's rule), so a continuation from ``prompt + partial
    output`` equals the uninterrupted one."""

    def __init__(self, vocab_size: int = 1000, max_batch: int = 64, max_ctx: int = 4096, num_blocks: int = 1 << 20,
                 step_delay_s: float = 0.0, fail_on: Optional[Callable[[str, List[str]], bool]] = None):
        self.vocab_size, self.max_batch, self.max_ctx, self.num_blocks = vocab_size, max_batch, max_ctx, num_blocks
        self.step_delay_s = step_delay_s
        self.fail_on = fail_on
        self.held: Dict[str, int] = {}
        self.calls: List[tuple] = []

    def _next(self, seq):
        from connex.serving.fake_backend import next_token
        return next_token(seq, self.vocab_size)

    def _step(self, kind, rids, seqs):
        self.calls.append((kind, list(rids)))
        if self.fail_on is not None and self.fail_on(kind, rids):
            raise RuntimeError(f"injected {kind} failure")
        if self.step_delay_s:
            time.sleep(self.step_delay_s)
        for r, s in zip(rids, seqs):
            self.held[r] = len(s)
        return [self._next(s) for s in seqs]

    supports_mixed = True

    def prefill(self, rids, seqs):
        return self._step("prefill", rids, seqs)

    def decode(self, rids, seqs):
        for r, s in zip(rids, seqs):
            assert self.held.get(r) == len(s) - 1, f"{r}: KV holds {self.held.get(r)}, sequence {len(s)}"
        return self._step("decode", rids, seqs)

    def mixed(self, rids, seqs, ctx, n_new):
        for r, c in zip(rids, ctx):
            assert self.held.get(r, 0) == c, f"{r}: KV holds {self.held.get(r)}, step continues at {c}"
        # named like the runtime's step kinds: all one-token rows run as a
        # decode step, fresh whole prompts as a prefill step
        kind = ("decode" if all(n == 1 for n in n_new) else
                "prefill" if not any(ctx) and all(n != 1 for n in n_new) else "mixed")
        return self._step(kind, rids, [s[:c + n] for s, c, n in zip(seqs, ctx, n_new)])

    def release(self, rids):
        for r in rids:
            self.held.pop(r, None)


class RuleStageRuntime:
    """CPU stand-in for one pipeline stage's compute (the step protocol of
    :class:`connex_b200.runtime.pp.StageRuntime`): the "activations" are the
    token ids themselves, every stage keeps each request's ids as its "KV"
    (so a replica that never saw a request lacks it and the rows come back
    missing), and the last stage answers the :class:`RuleStepper` rule.
    ``delay_s`` slows each step, to kill a replica mid-stream in tests."""

    def __init__(self, first: bool, last: bool, vocab_size: int = 1000, delay_s: float = 0.0):
        import torch
        self.first, self.last, self.vocab, self.delay_s = first, last, vocab_size, delay_s
        self.device = torch.device("cpu")
        self.seqs: Dict[str, List[int]] = {}
        self.steps = 0

    def kv_held(self, rid) -> int:
        return len(self.seqs.get(rid, ()))

    def release(self, rids) -> None:
        for r in rids:
            self.seqs.pop(r, None)

    def reprefill(self, rids) -> None:
        pass

    def abort(self, rids) -> None:
        self.release(rids)

    def compute(self, td: dict, missing) -> dict:
        import torch
        from connex.pp.handover import CX_CTX, REQUEST_IDS
        if td.get("kind") == "warmup":
            return {"kind": "warmup", "w": td["w"].clone()}
        if self.delay_s:
            time.sleep(self.delay_s)
        from connex.serving.fake_backend import next_token
        rids, ctx, n_new = list(td[REQUEST_IDS]), list(td[CX_CTX]), list(td["n_new"])
        x = (td["ids"] if self.first else td["x"]).to(torch.int64).tolist()
        i, nxt = 0, []
        for r, c, n in zip(rids, ctx, n_new):
            seq = [] if (c == 0 or r in missing) else self.seqs.get(r, [])[:c]
            seq = seq + x[i:i + n]
            i += n
            if r not in missing:
                self.seqs[r] = seq
            nxt.append(next_token(seq, self.vocab))
        self.steps += 1
        out = {"kind": td["kind"], "n_new": n_new}
        if "n_dec" in td:
            out["n_dec"] = td["n_dec"]
        if self.last:
            out["next"] = torch.tensor(nxt, dtype=torch.int64)
        else:
            out["x"] = torch.tensor(x, dtype=torch.int64)
        return out


class _RuntimeSteps(Stepper):
    """Step tensors for a :class:`connex_b200.runtime.pp.StageRuntime`."""

    supports_mixed = True

    def _td_rows(self, rids, seqs, ctx, n_new):
        """A mixed step: one-token rows first (decode attention), chunks after
        (the paged prefill kernel); pure decode / fresh prefill steps keep
        their own kinds (decode graphs, the contiguous prefill kernel).
        Returns (td, order) -- ``order[i]``: the caller's row at position i."""
        import torch
        from connex.pp.handover import CX_CTX, REQUEST_IDS
        order = sorted(range(len(rids)), key=lambda i: n_new[i] != 1)
        n_dec = sum(1 for n in n_new if n == 1)
        if n_dec == len(rids):
            kind = "decode"
        elif n_dec == 0 and not any(ctx):
            kind = "prefill"
        else:
            kind = "mixed"
        ids = [t for i in order for t in seqs[i][ctx[i]:ctx[i] + n_new[i]]]
        t = torch.tensor(ids, dtype=torch.int32)
        if self.rt.device.type == "cuda":
            t = t.pin_memory().to(self.rt.device, non_blocking=True)
        td = {"kind": kind, REQUEST_IDS: [rids[i] for i in order], CX_CTX: [ctx[i] for i in order],
              "n_new": [n_new[i] for i in order], "ids": t}
        if kind == "mixed":
            td["n_dec"] = n_dec
        return td, order

    @staticmethod
    def _unorder(order, vals):
        out = [0] * len(order)
        for pos, i in enumerate(order):
            out[i] = vals[pos]
        return out

    def _td(self, kind, rids, seqs):
        import torch
        from connex.pp.handover import CX_CTX, REQUEST_IDS
        if kind == "prefill":
            ids, ctx, n_new = [t for s in seqs for t in s], [0] * len(seqs), [len(s) for s in seqs]
        else:
            ids, ctx, n_new = [s[-1] for s in seqs], [len(s) - 1 for s in seqs], [1] * len(seqs)
        t = torch.tensor(ids, dtype=torch.int32)
        if self.rt.device.type == "cuda":
            t = t.pin_memory().to(self.rt.device, non_blocking=True)
        return {"kind": kind, REQUEST_IDS: list(rids), CX_CTX: ctx, "n_new": n_new, "ids": t}, ctx, n_new

    def release(self, rids):
        self.rt.release(list(rids))


def _make_runtime(cfg, l0, l1, device, num_blocks, max_batch, max_ctx, max_step_tokens, checkpoint, seed, tp=None):
    """A StageRuntime for layers [l0, l1); with ``tp`` (a TPGroup) this rank's
    shard of them (checkpoint shards are cut on the host; random weights are
    drawn whole and cut, so every TP degree serves the same model)."""
    from connex_b200.runtime.pp import StageRuntime, stage_weights
    weights, rcfg = None, cfg
    if checkpoint:
        from connex_b200.models.hf import load_llama
        weights = load_llama(checkpoint, device, layers=(l0, l1), cfg=cfg,
                             tp=(tp.rank, tp.world) if tp is not None else None)
        rcfg = weights.cfg
    elif tp is not None and tp.world > 1:
        from connex_b200.parallel.tp import shard_layer, tp_config
        full = stage_weights(cfg, l0, l1, device, seed)
        full.layers = [shard_layer(lw, cfg, tp.rank, tp.world) for lw in full.layers]
        full.cfg = rcfg = tp_config(cfg, tp.world)
        weights = full
    return StageRuntime(rcfg, l0, l1, device, num_blocks=num_blocks, max_tokens=max_step_tokens, max_batch=max_batch,
                        max_ctx=max_ctx, seed=seed, weights=weights, tp=tp)


class ModelStepper(_RuntimeSteps):
    """All layers on one GPU; decode steps replay CUDA graphs (``graphs``)."""

    def __init__(self, cfg, device, num_blocks: int, max_batch: int = 64, max_ctx: int = 4096,
                 max_step_tokens: int = 8192, checkpoint: Optional[str] = None, seed: int = 0, graphs: bool = True,
                 tp=None):
        self.cfg = cfg
        self.max_batch, self.max_ctx, self.max_step_tokens = max_batch, max_ctx, max_step_tokens
        self.block_size, self.vocab_size = cfg.block_size, cfg.vocab_size
        self.rt = _make_runtime(cfg, 0, cfg.layers, device, num_blocks, max_batch, max_ctx, max_step_tokens,
                                checkpoint, seed, tp)
        if graphs:
            self.rt.enable_decode_graphs()
        self.num_blocks = self.rt.cache.free_blocks          # less the graphs' trash block

    def _run(self, kind, rids, seqs):
        td, _, _ = self._td(kind, rids, seqs)
        return self.rt.compute(td, [])["next"].tolist()

    def prefill(self, rids, seqs):
        return self._run("prefill", rids, seqs)

    def decode(self, rids, seqs):
        return self._run("decode", rids, seqs)

    def mixed(self, rids, seqs, ctx, n_new):
        td, order = self._td_rows(rids, seqs, ctx, n_new)
        return self._unorder(order, self.rt.compute(td, [])["next"].tolist())


class GroupStepError(RuntimeError):
    """A step failed on one rank of a tensor-parallel group.  The ranks no
    longer issue matching collectives, so the whole group must stop: the
    engine treats this error as fatal (it fails every request and stops
    admitting new ones) instead of failing only the step's requests."""


class TPStepper(Stepper):
    """Rank 0 of a tensor-parallel group: every step (and every release) is
    broadcast to the other ranks over a CPU process group before it runs
    here, so all ranks launch the same kernels and the same all-reduces in
    the same order; the other ranks run :func:`tp_follow`.

    A failure anywhere is fatal to the group.  If this rank's step raises,
    the followers may be inside that step's all-reduces (or past them), so no
    later step can pair its collectives correctly: the stepper turns broken,
    tells the followers to exit (best effort, from a daemon thread so a
    follower stuck in a collective cannot block this rank) and raises
    :class:`GroupStepError`, which stops the engine.  If a follower's step
    raises, it exits; this rank's next collective then fails with the
    process group's timeout, which lands here the same way."""

    def __init__(self, inner: Stepper, cpu_group=None, src: int = 0):
        self.inner, self.pg, self.src = inner, cpu_group, src
        self.broken: Optional[str] = None
        self._abort_thread = None
        for k in ("max_batch", "max_ctx", "max_step_tokens", "num_blocks", "block_size", "vocab_size",
                  "supports_mixed"):
            setattr(self, k, getattr(inner, k))

    def _send(self, msg) -> None:
        import torch.distributed as dist
        if self.broken is not None:
            raise GroupStepError(f"tensor-parallel group is down: {self.broken}")
        dist.broadcast_object_list([msg], src=self.src, group=self.pg)

    def _fail(self, e: BaseException) -> GroupStepError:
        import threading as _th

        import torch.distributed as dist
        self.broken = f"{type(e).__name__}: {e}"

        def tell():
            try:
                dist.broadcast_object_list([("abort", self.broken)], src=self.src, group=self.pg)
            except Exception:  # noqa: BLE001 - the followers may be gone or stuck; nothing more to do
                pass
        self._abort_thread = _th.Thread(target=tell, name="cx-tp-abort", daemon=True)
        self._abort_thread.start()
        return GroupStepError(f"step failed on rank {self.src}; the tensor-parallel group stops: {self.broken}")

    def _run(self, kind, rids, seqs, *extra):
        if self.broken is not None:
            raise GroupStepError(f"tensor-parallel group is down: {self.broken}")
        try:
            self._send((kind, list(rids), [list(x) for x in seqs]) + tuple(list(e) for e in extra))
            return getattr(self.inner, kind)(rids, seqs, *extra)
        except Exception as e:  # noqa: BLE001 - any failure breaks collective matching
            raise self._fail(e) from e

    def prefill(self, rids, seqs):
        return self._run("prefill", rids, seqs)

    def decode(self, rids, seqs):
        return self._run("decode", rids, seqs)

    def mixed(self, rids, seqs, ctx, n_new):
        return self._run("mixed", rids, seqs, ctx, n_new)

    def release(self, rids):
        if self.broken is not None:
            return
        try:
            self._send(("release", list(rids)))
        except Exception as e:  # noqa: BLE001
            raise self._fail(e) from e
        self.inner.release(rids)

    def close(self):
        if self.broken is None:
            try:
                self._send(("stop",))
            except Exception:  # noqa: BLE001 - the followers are gone; close this rank anyway
                pass
        elif self._abort_thread is not None:
            # give the abort notice a bounded chance to reach the followers
            # before this rank's process group can be torn down under it
            self._abort_thread.join(timeout=5.0)
        self.inner.close()


def tp_follow(inner: Stepper, cpu_group=None, src: int = 0) -> int:
    """Ranks 1.. of a tensor-parallel group: run rank ``src``'s steps until it
    stops; returns the number of steps run.  Raises :class:`GroupStepError`
    when rank ``src`` reports a failed step; a step failing here propagates
    (the caller exits, and rank ``src``'s next collective fails)."""
    import torch.distributed as dist
    n = 0
    while True:
        box = [None]
        dist.broadcast_object_list(box, src=src, group=cpu_group)
        msg = box[0]
        if msg[0] == "stop":
            inner.close()
            return n
        if msg[0] == "abort":
            inner.close()
            raise GroupStepError(f"rank {src} failed a step: {msg[1]}")
        if msg[0] == "release":
            inner.release(msg[1])
        else:
            getattr(inner, msg[0])(*msg[1:])
            n += 1


class _Stage0Hooks:
    def __init__(self):
        self.reprefill_rids: List[str] = []

    def kv_held(self, rid):
        return 0

    def release(self, rids):
        pass

    def reprefill(self, rids):
        self.reprefill_rids = list(rids)

    def abort(self, rids):
        pass


class PipelineStepper(_RuntimeSteps):
    """Stage 0 of a pipeline: layers ``[0, l1)`` here, the rest downstream
    through ``endpoint`` (a :class:`connex.pp.endpoint.PipelineEndpoint` with
    membership attached).  Downstream stages serve the same step protocol
    with :class:`connex_b200.runtime.pp.StageRuntime` (``python -m
    connex_b200.serve.stage``)."""

    def __init__(self, cfg, l1: int, device, endpoint, num_blocks: int, max_batch: int = 64, max_ctx: int = 4096,
                 max_step_tokens: int = 8192, checkpoint: Optional[str] = None, seed: int = 0,
                 recv_timeout_s: float = 30.0, graphs: bool = True, rt=None):
        """``rt``: stage 0's compute when not the Llama runtime (the CPU
        stand-in :class:`RuleStageRuntime`)."""
        from connex.pp.link import Stage0Link
        self.cfg = cfg
        self.max_batch, self.max_ctx, self.max_step_tokens = max_batch, max_ctx, max_step_tokens
        self.block_size, self.vocab_size = cfg.block_size, cfg.vocab_size
        self.rt = rt if rt is not None else _make_runtime(cfg, 0, l1, device, num_blocks, max_batch, max_ctx,
                                                          max_step_tokens, checkpoint, seed)
        if graphs and rt is None:
            self.rt.enable_decode_graphs()
        # downstream stages keep a trash block too when they run graphs
        self.num_blocks = num_blocks - 1
        self.ep = endpoint
        self.hooks = _Stage0Hooks()
        self.link = Stage0Link(endpoint, self.hooks, recv_timeout_s=recv_timeout_s)
        self.reprefills = 0

    def _through(self, td, rids, ctx, n_new):
        """This stage's layers, then the rest of the pipeline; the next ids."""
        x = self.rt.compute(td, [])["x"]
        self.hooks.reprefill_rids = []
        step = {"x": x, "kind": td["kind"], "n_new": n_new}
        if "n_dec" in td:
            step["n_dec"] = td["n_dec"]
        return self.link.step(step, request_ids=list(rids), num_computed=ctx)["next"].tolist()

    def _repair(self, rids, seqs, upto, nxt):
        """Rows whose KV the new downstream replica lacks: read their
        sequences up to ``upto`` again through the whole pipeline (in chunks
        of the step budget); the last position's id replaces this step's."""
        again = list(self.hooks.reprefill_rids)
        if not again:
            return nxt
        self.reprefills += len(again)
        idx = [list(rids).index(r) for r in again]
        self.rt.release(again)
        done = [0] * len(idx)
        while True:
            rows = [j for j, i in enumerate(idx) if done[j] < upto[i]]
            if not rows:
                return nxt
            budget, take = self.max_step_tokens, []
            for j in rows:
                n = min(upto[idx[j]] - done[j], budget)
                if n <= 0:
                    break
                take.append((j, n))
                budget -= n
            sub_r = [again[j] for j, _ in take]
            sub_s = [seqs[idx[j]] for j, _ in take]
            sub_c = [done[j] for j, _ in take]
            sub_n = [n for _, n in take]
            td, order = self._td_rows(sub_r, sub_s, sub_c, sub_n)
            got = self._unorder(order, self._through(td, td[REQUEST_IDS], td[CX_CTX], td["n_new"]))
            for (j, n), tok in zip(take, got):
                done[j] += n
                if done[j] == upto[idx[j]]:
                    nxt[idx[j]] = tok

    def _run(self, kind, rids, seqs):
        td, ctx, n_new = self._td(kind, rids, seqs)
        nxt = self._through(td, rids, ctx, n_new)
        return self._repair(rids, seqs, [len(s) for s in seqs], nxt)

    def prefill(self, rids, seqs):
        return self._run("prefill", rids, seqs)

    def decode(self, rids, seqs):
        return self._run("decode", rids, seqs)

    def mixed(self, rids, seqs, ctx, n_new):
        td, order = self._td_rows(rids, seqs, ctx, n_new)
        nxt = self._unorder(order, self._through(td, td[REQUEST_IDS], td[CX_CTX], td["n_new"]))
        return self._repair(rids, seqs, [c + n for c, n in zip(ctx, n_new)], nxt)

    def release(self, rids):
        self.rt.release(list(rids))
        self.link.finished(list(rids))          # downstream stages free them on the next steps

    def close(self):
        self.ep.close()


@dataclass
class Request:
    rid: str
    prompt: List[int]
    max_tokens: int
    on_token: Callable[["Request", Optional[int], Optional[str]], None]
    stop_ids: frozenset = frozenset()
    gen: List[int] = field(default_factory=list)
    done: int = 0                  # prompt tokens already in the KV cache (chunked prefill)
    blocks: int = 0
    cancelled: bool = False
    finish_reason: Optional[str] = None
    error: Optional[str] = None
    t_submit: float = field(default_factory=time.monotonic)
    t_first: Optional[float] = None


class EngineFull(Exception):
    """The request can never fit (context or KV capacity)."""


class GenerationEngine:
    """Scheduler thread over a :class:`Stepper` (see the module docstring).

    ``on_token(req, token, finish_reason)`` is called from the engine thread
    once per generated token (``finish_reason`` set on the last one), or
    with ``token=None`` and a reason (``"error"`` / ``"abort"``) when the
    request ends without one."""

    def __init__(self, stepper: Stepper, max_batch: Optional[int] = None, max_step_tokens: Optional[int] = None,
                 idle_wait_s: float = 0.05, chunked: Optional[bool] = None):
        self.s = stepper
        self.max_batch = max_batch or stepper.max_batch
        self.max_step_tokens = max_step_tokens or stepper.max_step_tokens
        self.chunked = bool(getattr(stepper, "supports_mixed", False)) if chunked is None else chunked
        self.idle_wait_s = idle_wait_s
        self.waiting: "collections.deque[Request]" = collections.deque()
        self.running: Dict[str, Request] = {}
        self.blocks_reserved = 0
        self._cv = threading.Condition()
        self._stop = threading.Event()
        self._ids = itertools.count()
        self.stats = collections.Counter()
        self.error: Optional[str] = None
        self._thread: Optional[threading.Thread] = None

    # ------------------------------------------------------------ client side
    def blocks_for(self, n_tokens: int) -> int:
        return -(-n_tokens // self.s.block_size)

    def submit(self, prompt: Sequence[int], max_tokens: int, on_token, stop_ids=(), rid: Optional[str] = None
               ) -> Request:
        prompt = [int(t) for t in prompt]
        if not prompt:
            raise ValueError("empty prompt")
        if max_tokens <= 0:
            raise ValueError("max_tokens must be positive")
        if self.error is not None:
            raise EngineFull(f"engine stopped: {self.error}")
        if len(prompt) + max_tokens > self.s.max_ctx:
            raise EngineFull(f"prompt ({len(prompt)}) + max_tokens ({max_tokens}) exceeds the context "
                             f"({self.s.max_ctx})")
        if len(prompt) > self.max_step_tokens and not self.chunked:
            raise EngineFull(f"prompt ({len(prompt)}) exceeds the prefill budget ({self.max_step_tokens})")
        if self.s.vocab_size and any(not 0 <= t < self.s.vocab_size for t in prompt):
            raise ValueError(f"token ids must lie in [0, {self.s.vocab_size})")
        blocks = self.blocks_for(len(prompt) + max_tokens)
        if blocks > self.s.num_blocks:
            raise EngineFull(f"request needs {blocks} KV blocks, the cache has {self.s.num_blocks}")
        req = Request(rid or f"r{next(self._ids)}", prompt, int(max_tokens), on_token, frozenset(stop_ids or ()),
                      blocks=blocks)
        with self._cv:
            self.waiting.append(req)
            self.stats["submitted"] += 1
            self._cv.notify()
        return req

    def cancel(self, req: Request) -> None:
        req.cancelled = True
        with self._cv:
            self._cv.notify()

    def start(self) -> "GenerationEngine":
        self._thread = threading.Thread(target=self._loop, name="cx-serve-engine", daemon=True)
        self._thread.start()
        return self

    def stop(self, timeout: float = 10.0) -> None:
        self._stop.set()
        with self._cv:
            self._cv.notify()
        if self._thread is not None:
            self._thread.join(timeout)

    @property
    def alive(self) -> bool:
        return self._thread is not None and self._thread.is_alive() and self.error is None

    def load(self) -> dict:
        with self._cv:
            return {"waiting": len(self.waiting), "running": len(self.running),
                    "kv_blocks_reserved": self.blocks_reserved, "kv_blocks": self.s.num_blocks}

    # ------------------------------------------------------------ engine thread
    def _finish(self, reqs: List[Request], reason: str, token_sent: bool = True) -> None:
        rel = [r.rid for r in reqs if r.rid in self.running]
        for r in reqs:
            if self.running.pop(r.rid, None) is not None:
                self.blocks_reserved -= r.blocks
            r.finish_reason = reason
            self.stats["finished_" + reason] += 1
            if not token_sent:
                try:
                    r.on_token(r, None, reason)
                except Exception:  # noqa: BLE001 - a broken callback must not stop the engine
                    log.exception("callback of %s", r.rid)
        if rel:
            self.s.release(rel)

    def _admit(self) -> List[Request]:
        new, tokens = [], 0
        with self._cv:
            while self.waiting:
                r = self.waiting[0]
                if r.cancelled:
                    self.waiting.popleft()
                    r.finish_reason = "abort"
                    self.stats["finished_abort"] += 1
                    continue
                if len(self.running) + len(new) >= self.max_batch:
                    break
                if not self.chunked and new and tokens + len(r.prompt) > self.max_step_tokens:
                    break
                if self.blocks_reserved + r.blocks > self.s.num_blocks:
                    break
                self.waiting.popleft()
                self.blocks_reserved += r.blocks
                tokens += len(r.prompt)
                new.append(r)
        return new

    def _emit(self, reqs: List[Request], toks: List[int]) -> None:
        done = collections.defaultdict(list)
        now = time.monotonic()
        for r, t in zip(reqs, toks):
            r.gen.append(int(t))
            if r.t_first is None:
                r.t_first = now
            reason = None
            if int(t) in r.stop_ids:
                reason = "stop"
            elif len(r.gen) >= r.max_tokens:
                reason = "length"
            self.stats["tokens"] += 1
            try:
                r.on_token(r, int(t), reason)
            except Exception:  # noqa: BLE001
                log.exception("callback of %s", r.rid)
                reason = reason or "abort"
            if reason:
                done[reason].append(r)
        for reason, rs in done.items():
            self._finish(rs, reason)

    def _step(self, kind: str, reqs: List[Request]) -> None:
        rids = [r.rid for r in reqs]
        seqs = [r.prompt + r.gen for r in reqs]
        try:
            toks = (self.s.prefill if kind == "prefill" else self.s.decode)(rids, seqs)
        except GroupStepError:
            raise                       # fatal: the loop ends and fails every request
        except Exception as e:  # noqa: BLE001 - fail the step's requests, keep serving
            log.exception("%s step of %d requests failed", kind, len(reqs))
            self.stats["step_errors"] += 1
            for r in reqs:
                r.error = f"{type(e).__name__}: {e}"
            self._finish(reqs, "error", token_sent=False)
            return
        self.stats[kind + "_steps"] += 1
        self._emit(reqs, toks)

    def _step_mixed(self) -> None:
        """One mixed step: a decode row per generating request, then prefill
        chunks of the prompts still being read, in admission order, within
        the step's token budget."""
        decode = [r for r in self.running.values() if r.done == len(r.prompt)]
        budget = max(0, self.max_step_tokens - len(decode))
        chunks = []
        for r in self.running.values():
            if r.done < len(r.prompt) and budget > 0:
                n = min(len(r.prompt) - r.done, budget)
                chunks.append((r, n))
                budget -= n
        reqs = decode + [r for r, _ in chunks]
        if not reqs:
            return
        seqs = [r.prompt + r.gen for r in decode] + [r.prompt for r, _ in chunks]
        ctx = [len(s) - 1 for s in seqs[:len(decode)]] + [r.done for r, _ in chunks]
        n_new = [1] * len(decode) + [n for _, n in chunks]
        try:
            toks = self.s.mixed([r.rid for r in reqs], seqs, ctx, n_new)
        except GroupStepError:
            raise
        except Exception as e:  # noqa: BLE001 - fail the step's requests, keep serving
            log.exception("mixed step of %d rows failed", len(reqs))
            self.stats["step_errors"] += 1
            for r in reqs:
                r.error = f"{type(e).__name__}: {e}"
            self._finish(reqs, "error", token_sent=False)
            return
        # steps named like the runtime's kinds: one-token rows only, chunks only, or both
        self.stats["decode_steps" if not chunks else "prefill_steps" if not decode else "mixed_steps"] += 1
        self.stats["chunks"] += len(chunks)
        first = []
        for (r, n), tok in zip(chunks, toks[len(decode):]):
            r.done += n
            if r.done == len(r.prompt):
                first.append((r, tok))       # its last chunk: the first generated token
        self._emit(decode + [r for r, _ in first], toks[:len(decode)] + [t for _, t in first])

    def _loop(self) -> None:
        try:
            while not self._stop.is_set():
                gone = [r for r in self.running.values() if r.cancelled]
                if gone:
                    self._finish(gone, "abort", token_sent=False)
                new = self._admit()
                if not new and not self.running:
                    with self._cv:
                        if not self.waiting and not self._stop.is_set():
                            self._cv.wait(self.idle_wait_s)
                    continue
                if self.chunked:
                    for r in new:
                        self.running[r.rid] = r
                    self._step_mixed()
                    continue
                decoding = list(self.running.values())
                if new:
                    for r in new:
                        self.running[r.rid] = r
                    self._step("prefill", new)
                decoding = [r for r in decoding if r.rid in self.running]
                if decoding:
                    self._step("decode", decoding)
        except Exception as e:  # noqa: BLE001
            log.exception("engine loop died")
            self.error = f"{type(e).__name__}: {e}"
        finally:
            with self._cv:
                left = list(self.running.values()) + list(self.waiting)
                self.waiting.clear()
            self._finish(left, "abort", token_sent=False)
